// SPDX-License-Identifier: Apache-2.0
// Host-side helpers shared by the pipelines: device selection, stream-ordered scratch buffers and
// the read-back checks of the range flags and the GEMM wait-timeout word.
#pragma once
#include <algorithm>
#include <string>

#include "oztt_common.cuh"

namespace oztt {

// Selects the device, checks that it is a B200-class GPU (compute capability 10.0) and keeps the
// stream-ordered pool's memory between calls.
void open_device(int device_id);
// Throws runtime_error for a GEMM wait timeout or for range flags of the scaling stage.
void check_flags(uint32_t flags, int gemm_err);

// Stream-ordered device buffer, released on the stream when it goes out of scope.
struct DevBuf {
    void* p = nullptr;
    cudaStream_t st;
    explicit DevBuf(cudaStream_t s) : st(s) {}
    DevBuf(cudaStream_t s, size_t bytes) : st(s) { alloc(bytes); }
    ~DevBuf() {
        if (p) cudaFreeAsync(p, st);
    }
    void alloc(size_t bytes) {
        const cudaError_t e = cudaMallocAsync(&p, std::max<size_t>(bytes, 256), st);
        if (e != cudaSuccess) {
            cudaGetLastError();
            p = nullptr;
            throw Error(OZTT_ERUNTIME, "device memory allocation of " + std::to_string(bytes) +
                                           " bytes failed: " + cudaGetErrorString(e));
        }
    }
    template <class T>
    T* as() const {
        return reinterpret_cast<T*>(p);
    }
    DevBuf(const DevBuf&) = delete;
    DevBuf& operator=(const DevBuf&) = delete;
};


}  // namespace oztt
