// TEST INFRASTRUCTURE. Stand-ins for the three TT-Metalium names that the reference's host
// planner headers use (src/backend/common/format.hpp:24-131), so that the planner compiles
// in place on a machine without TT-Metalium. Only the names and the tile sizes matter here.
#pragma once
#include <cstdint>
namespace tt {
enum class DataFormat { Int8, UInt8, Int32, Fp8_e4m3, Float32, Float16_b, Float16, UInt16, Bfp8_b, Bfp4_b, Bfp2_b };
constexpr uint32_t tile_size(DataFormat f) {
    switch (f) {
    case DataFormat::Int8: case DataFormat::UInt8: case DataFormat::Fp8_e4m3: return 1024;
    case DataFormat::Int32: case DataFormat::Float32: return 4096;
    case DataFormat::Float16_b: case DataFormat::Float16: case DataFormat::UInt16: return 2048;
    case DataFormat::Bfp8_b: return 1088;
    case DataFormat::Bfp4_b: return 576;
    case DataFormat::Bfp2_b: return 320;
    }
    return 0;
}
namespace tt_metal {
enum class MathFidelity { LoFi, HiFi2, HiFi3, HiFi4 };
}
}  // namespace tt
