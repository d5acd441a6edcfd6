// Gather kernel: copies compressed units into one contiguous slab.
//
// The reference packs a store job's payloads with torch.cat on the GPU and
// one D2H copy (vllm_v1_compressed_offload.py:371-447); this is the same
// step as one launch.  Units start at `align`-byte boundaries of the slab so
// that a restore can decode them in place after one H2D copy.
#include "ckv_launch.h"

namespace ckv {
namespace {

constexpr uint32_t kChunk = 64 * 1024;  // bytes per CTA

__global__ void __launch_bounds__(kThreads) pack_kernel(const PackUnit* units,
                                                        uint32_t count, uint8_t* dst) {
    for (uint32_t u = blockIdx.y; u < count; u += gridDim.y) {
        const PackUnit p = units[u];
        const uint64_t begin = static_cast<uint64_t>(blockIdx.x) * kChunk;
        if (begin >= p.size) continue;
        const uint64_t end = min(begin + kChunk, p.size);
        const uint8_t* src = p.src + begin;
        uint8_t* out = dst + p.offset + begin;
        const uint64_t len = end - begin;
        if (((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(out)) & 15u) == 0) {
            const uint64_t vec = len / 16;
            const uint4* s4 = reinterpret_cast<const uint4*>(src);
            uint4* d4 = reinterpret_cast<uint4*>(out);
            for (uint64_t i = threadIdx.x; i < vec; i += kThreads) d4[i] = __ldg(s4 + i);
            for (uint64_t i = vec * 16 + threadIdx.x; i < len; i += kThreads) out[i] = src[i];
        } else {
            for (uint64_t i = threadIdx.x; i < len; i += kThreads) out[i] = src[i];
        }
    }
}

// Descriptor upload: copies `words` 16-byte words from mapped page-locked
// host memory (read over PCIe by the SMs) into device memory, one word per
// thread so that the whole copy is one PCIe round trip.  A host-to-device
// cudaMemcpyAsync would queue on a copy engine behind any large
// host-to-device copy in flight on another stream; this does not.
__global__ void __launch_bounds__(kThreads) fetch_kernel(const uint4* src, uint4* dst,
                                                         uint32_t words) {
    const uint32_t i = blockIdx.x * kThreads + threadIdx.x;
    if (i < words) dst[i] = src[i];
}

}  // namespace

cudaError_t launch_fetch(const void* mapped_src, void* dst, size_t bytes, cudaStream_t stream) {
    if (bytes == 0) return cudaSuccess;
    if ((bytes & 15u) || ((reinterpret_cast<uintptr_t>(mapped_src) |
                           reinterpret_cast<uintptr_t>(dst)) & 15u))
        return cudaErrorInvalidValue;
    const uint32_t words = static_cast<uint32_t>(bytes / 16);
    note_launch();
    fetch_kernel<<<(words + kThreads - 1) / kThreads, kThreads, 0, stream>>>(
        static_cast<const uint4*>(mapped_src), static_cast<uint4*>(dst), words);
    return cudaGetLastError();
}

cudaError_t launch_pack(const PackUnit* units, uint32_t count, uint64_t max_size,
                        uint8_t* dst, cudaStream_t stream) {
    if (count == 0) return cudaSuccess;
    const uint64_t chunks = (max_size + kChunk - 1) / kChunk;
    dim3 grid(static_cast<uint32_t>(chunks ? chunks : 1), count < 65535u ? count : 65535u, 1);
    note_launch();
    pack_kernel<<<grid, kThreads, 0, stream>>>(units, count, dst);
    return cudaGetLastError();
}

}  // namespace ckv
