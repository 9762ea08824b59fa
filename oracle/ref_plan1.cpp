// TEST INFRASTRUCTURE — checker only, never shipped.
//
// Compiles the reference's Scheme I slice-count selection (src/backend/ozaki1/auto_precision.hpp,
// oz_fp64_p, with common/norm_estimate.hpp, common/bits.hpp and common/kernels/scale_bits.h) in place
// and exposes it through a C ABI, so that tests can compare the project's selection with the
// reference's on the same inputs. ref_shim1/ozaki1/format.hpp supplies the INT8 constants without the
// device API. Built by oracle/Makefile (target ref) into oracle/_ref/.
#include <cstdint>
#include <vector>

#include "ozaki1/auto_precision.hpp"

namespace r1 = ozTTgemm::detail::ozaki1_x;

extern "C" int ozr_i_slices(const double* a, const double* b, uint32_t M, uint32_t N, uint32_t K) {
    const std::vector<double> A(a, a + (size_t)M * K), B(b, b + (size_t)K * N);
    return r1::oz_fp64_p(A, B, M, N, K);
}
