// TEST INFRASTRUCTURE — checker only, never shipped.
//
// Stands in for src/backend/ozaki1/format.hpp when oracle/ref_plan1.cpp compiles the reference's
// ozaki1/auto_precision.hpp in place: that header needs only the four format constants below, while the
// real format.hpp pulls in the TT-Metalium device API. The values are the ones the real header derives
// for OZ_FMT_ID == INT8 (ozaki1/param.hpp:47 radix 254; digit bound radix/2; target 2^-1; maxima
// rounded up to BF16, CEIL mode 1), or for FP8 when OZ_FMT_FP8 is defined.
#pragma once
#include <cstdint>

namespace ozTTgemm::detail::OZTTGEMM_BACKEND_NS {
#if defined(OZ_FMT_FP8)
// FP8 (ozaki1/param.hpp:50 radix 32; digit bound 16 = min(radix/2, exact_int_max 16); target 2^-1;
// maxima truncated to BF16, CEIL mode 0, because the span 16/31 exceeds 2^-1 by more than 1/128).
inline constexpr uint32_t OZ1_RADIX = 32;
inline constexpr uint32_t OZ1_DMAX = 16;
inline constexpr int32_t OZ1_NSHIFT = -1;
inline constexpr uint32_t OZ1_CEIL_MODE = 0;
#elif defined(OZ_FMT_BF16) || defined(OZ_FMT_FP16) || defined(OZ_FMT_FP32)
// BF16, FP16, TF32 (param.hpp:55-65 radix 64; digit bound 32; target 2^-1; maxima truncated to BF16,
// CEIL mode 0).
inline constexpr uint32_t OZ1_RADIX = 64;
inline constexpr uint32_t OZ1_DMAX = 32;
inline constexpr int32_t OZ1_NSHIFT = -1;
inline constexpr uint32_t OZ1_CEIL_MODE = 0;
#else
inline constexpr uint32_t OZ1_RADIX = 254;
inline constexpr uint32_t OZ1_DMAX = 127;
inline constexpr int32_t OZ1_NSHIFT = -1;
inline constexpr uint32_t OZ1_CEIL_MODE = 1;
#endif
}  // namespace ozTTgemm::detail::OZTTGEMM_BACKEND_NS
