// SPDX-License-Identifier: Apache-2.0
//
// ozTTgemm for NVIDIA B200: FP64 matrix multiplication by the Ozaki schemes on sm_100a.
//
// Drop-in public interface of mukunoki/ozTT's ozTTgemm (include/ozTTgemm/ozTTgemm.hpp:25-121 of the
// reference): the same types, members, defaults and functions. The FP64 operands are split into
// exactly multiplied int8 matrices (residues modulo small moduli for scheme II), the products run on
// the tensor cores, and the FP64 result is reconstructed on the GPU.
//
// Differences a caller can observe (the declarations are identical):
//   * Format::INT8, FP8 (e4m3 digits), BF16, FP16 and TF32 are built, both schemes.
//   * Format::BFP8, BFP4 and BFP2 are Tenstorrent block formats; is_available() is false for them, so a
//     default-constructed Options (format BFP8) is rejected with std::invalid_argument, exactly as the
//     reference rejects a format left out of its build.
//   * DeviceOptions::device_id is a CUDA device ordinal; kernel_directory is accepted and ignored (the
//     kernels are compiled into the library).
#pragma once

#include <cstddef>
#include <cstdint>
#include <memory>
#include <span>
#include <string>
#include <vector>

#define OZTTGEMM_VERSION_MAJOR 0
#define OZTTGEMM_VERSION_MINOR 1
#define OZTTGEMM_VERSION_PATCH 0

namespace ozTTgemm {

// Scheme I multiplies slice pairs; scheme II multiplies residues modulo several moduli (CRT).
enum class Scheme { I, II };

// Number format of the low-precision products.
enum class Format { BF16, FP16, TF32, BFP8, FP8, INT8, BFP4, BFP2 };

// Reconstruction passes of scheme II (Automatic: chosen from an error estimate of the input).
enum class Reconstruction { Automatic, OnePass, TwoPass };

// Options of the scheme that is not selected must keep their defaults.
struct Options {
    Scheme scheme = Scheme::II;
    Format format = Format::BFP8;
    // Scheme I only: 0 chooses the number of slices from the input, 1..256 fixes it.
    std::uint32_t slices = 0;
    // Scheme II only: 0 leaves the moduli to the library, 1..24 limits their number.
    std::uint32_t max_moduli = 0;
    // Scheme II only.
    Reconstruction reconstruction = Reconstruction::Automatic;
};

struct DeviceOptions {
    // CUDA device ordinal.
    int device_id = 0;
    // Kept for source compatibility; the B200 kernels are part of the library.
    std::string kernel_directory;
};

// What a call used.
struct Info {
    Scheme scheme;
    Format format;
    std::uint32_t slices = 0;                 // scheme I: number of slices
    std::uint32_t moduli = 0;                 // scheme II: number of CRT moduli
    std::uint32_t integer_bits = 0;           // scheme II: bits kept of each scaled operand
    std::uint32_t reconstruction_passes = 0;  // scheme II: 1 or 2
    // m and n rounded up to multiples of 64, k to a multiple of 32 (the planning dimensions).
    std::size_t padded_m = 0, padded_n = 0, padded_k = 0;
};

// False for formats this build does not provide.
bool is_available(Format format) noexcept;
// "BF16", "FP16", "TF32", "BFP8", "FP8", "INT8", "BFP4" or "BFP2".
const char* format_name(Format format) noexcept;

// Owns one CUDA device, initialised on the first valid GEMM. Calls of all contexts in a process
// are serialised. Intermediate device buffers are released after each call.
class Context {
public:
    // std::invalid_argument if device_id is negative.
    explicit Context(DeviceOptions options = {});
    ~Context();
    Context(const Context&) = delete;
    Context& operator=(const Context&) = delete;
    Context(Context&&) = delete;
    Context& operator=(Context&&) = delete;

    // C = A*B for contiguous row-major FP64 A[m,k], B[k,n], C[m,n]. The spans must hold exactly m*k,
    // k*n and m*n elements. All input is consumed before C is written, so C may overlap A or B.
    // Inputs must be finite and every nonzero row maximum of A and column maximum of B must lie in
    // [2^-126, largest finite BF16]. A result that would be subnormal is returned as zero.
    // Throws std::invalid_argument for invalid input (before the device is used and before C is
    // written), std::runtime_error for configurations that cannot be executed and for CUDA failures,
    // and std::bad_alloc if host memory runs out. The library never writes to stdout or stderr.
    Info gemm(std::span<const double> a, std::span<const double> b, std::span<double> c, std::size_t m, std::size_t n,
              std::size_t k, const Options& options = {});

    // Same as gemm(), returning C as a new vector.
    std::vector<double> multiply(std::span<const double> a, std::span<const double> b, std::size_t m, std::size_t n,
                                 std::size_t k, const Options& options = {});

private:
    struct Impl;
    std::unique_ptr<Impl> impl_;
};

}  // namespace ozTTgemm
