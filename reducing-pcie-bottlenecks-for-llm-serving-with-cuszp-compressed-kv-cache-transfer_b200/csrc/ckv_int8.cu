// INT8 page codec of the reference's comparison protocol, and page copies
// for its raw encoding, as kernels for the store / restore pipeline.
//
// INT8 (vllm_v1_compressed_offload.py:711-724 store, :2090-2116 restore):
//   scale = max|x| / 127.0 as the reference evaluates it on a CUDA tensor:
//     ATen divides a tensor by a CPU scalar as a multiply by the float32
//     reciprocal, max|x| * (1.0f / 127.0f), each rounded to nearest
//     (BinaryDivTrueKernel.cu); 1 when the page is all zeros;
//   q = clamp(round_half_even(x / scale), -127, 127) as int8,
//   restore: bf16_rn((float)q * scale).
// A stored page is its n int8 values followed by the FP32 scale at byte
// align4(n) (the reference keeps the scale beside the payload and counts
// numel + 4 bytes).  The page maximum is a separate pass: every CTA of a
// page folds its slice into one word with an atomic max of |x| as BF16 bits
// (non-negative BF16 values order like their bit patterns; a NaN sorts above
// infinity, so a page with a NaN gets a NaN scale as torch's max gives).
//
// Raw pages (:1578-1615) are byte copies: one launch gathers a chunk's pages
// into the staging buffer or scatters a landing buffer into the pages.
#include "ckv_launch.h"

namespace ckv {
namespace {

constexpr uint32_t kSliceElems = 16384;   // elements per CTA (32 KB of BF16)
constexpr uint64_t kCopyChunk = 64 * 1024;

constexpr float kInv127 = 1.0f / 127.0f;   // the float32 reciprocal, rounded to nearest

__device__ __forceinline__ float page_scale(uint32_t amax_bits) {
    const float scale = __fmul_rn(__uint_as_float(amax_bits << 16), kInv127);
    return scale == 0.0f ? 1.0f : scale;
}

// torch.clamp keeps a NaN quotient and the int8 cast turns it into 0 (a
// page with a NaN has a NaN scale, so every value of it is stored as 0).
__device__ __forceinline__ uint32_t quantise(float x, float scale) {
    const float v = rintf(__fdiv_rn(x, scale));
    const float q = v != v ? 0.0f : fminf(fmaxf(v, -127.0f), 127.0f);
    return static_cast<uint32_t>(static_cast<int32_t>(q)) & 0xffu;
}

__device__ __forceinline__ uint16_t dequantise(uint32_t byte, float scale) {
    const float x = __fmul_rn(static_cast<float>(static_cast<int8_t>(byte)), scale);
    return __bfloat16_as_ushort(__float2bfloat16_rn(x));
}

__global__ void __launch_bounds__(kThreads) absmax_kernel(const Int8Unit* units, uint32_t count) {
    for (uint32_t u = blockIdx.y; u < count; u += gridDim.y) {
        const Int8Unit d = units[u];
        const uint32_t e0 = blockIdx.x * kSliceElems;
        if (e0 >= d.n) continue;
        const uint32_t e1 = min(e0 + kSliceElems, d.n);
        const uint16_t* page = static_cast<const uint16_t*>(d.page);
        uint32_t m = 0;
        if ((reinterpret_cast<uintptr_t>(page) & 15u) == 0) {
            const uint32_t v1 = e0 + (e1 - e0) / 8 * 8;
            const uint4* p4 = reinterpret_cast<const uint4*>(page + e0);
            for (uint32_t i = threadIdx.x; i < (v1 - e0) / 8; i += kThreads) {
                const uint4 w = __ldg(p4 + i);
                const uint32_t a = __vmaxu2(w.x & 0x7fff7fffu, w.y & 0x7fff7fffu);
                const uint32_t b = __vmaxu2(w.z & 0x7fff7fffu, w.w & 0x7fff7fffu);
                const uint32_t c = __vmaxu2(a, b);
                m = max(m, max(c & 0xffffu, c >> 16));
            }
            for (uint32_t i = v1 + threadIdx.x; i < e1; i += kThreads) m = max(m, page[i] & 0x7fffu);
        } else {
            for (uint32_t i = e0 + threadIdx.x; i < e1; i += kThreads) m = max(m, page[i] & 0x7fffu);
        }
        m = __reduce_max_sync(0xffffffffu, m);
        if ((threadIdx.x & 31) == 0 && m) atomicMax(d.amax, m);
    }
}

__global__ void __launch_bounds__(kThreads) quant_kernel(const Int8Unit* units, uint32_t count) {
    for (uint32_t u = blockIdx.y; u < count; u += gridDim.y) {
        const Int8Unit d = units[u];
        const uint32_t e0 = blockIdx.x * kSliceElems;
        if (e0 >= d.n) continue;
        const uint32_t e1 = min(e0 + kSliceElems, d.n);
        const uint32_t amax = *reinterpret_cast<const volatile uint32_t*>(d.amax);
        const float scale = page_scale(amax);
        if (blockIdx.x == 0 && threadIdx.x == 0)
            *reinterpret_cast<float*>(d.q + align4(d.n)) = scale;
        const uint16_t* page = static_cast<const uint16_t*>(d.page);
        if (((reinterpret_cast<uintptr_t>(page) | reinterpret_cast<uintptr_t>(d.q)) & 15u) == 0) {
            // 16 elements per thread: two 16-byte loads, one 16-byte store
            const uint32_t v1 = e0 + (e1 - e0) / 16 * 16;
            for (uint32_t i = e0 / 16 + threadIdx.x; i < v1 / 16; i += kThreads) {
                const uint4* p4 = reinterpret_cast<const uint4*>(page) + 2 * i;
                const uint4 a = __ldg(p4), b = __ldg(p4 + 1);
                const uint32_t in[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
                uint32_t out[4];
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const uint32_t w0 = in[2 * k], w1 = in[2 * k + 1];
                    out[k] = quantise(bf16_lo(w0), scale) | quantise(bf16_hi(w0), scale) << 8 |
                             quantise(bf16_lo(w1), scale) << 16 | quantise(bf16_hi(w1), scale) << 24;
                }
                reinterpret_cast<uint4*>(d.q)[i] = make_uint4(out[0], out[1], out[2], out[3]);
            }
            for (uint32_t i = v1 + threadIdx.x; i < e1; i += kThreads)
                d.q[i] = static_cast<uint8_t>(quantise(__uint_as_float(uint32_t(page[i]) << 16), scale));
        } else {
            for (uint32_t i = e0 + threadIdx.x; i < e1; i += kThreads)
                d.q[i] = static_cast<uint8_t>(quantise(__uint_as_float(uint32_t(page[i]) << 16), scale));
        }
    }
}

__global__ void __launch_bounds__(kThreads) dequant_kernel(const Int8Unit* units, uint32_t count) {
    for (uint32_t u = blockIdx.y; u < count; u += gridDim.y) {
        const Int8Unit d = units[u];
        const uint32_t e0 = blockIdx.x * kSliceElems;
        if (e0 >= d.n) continue;
        const uint32_t e1 = min(e0 + kSliceElems, d.n);
        const float scale = *reinterpret_cast<const float*>(d.q + align4(d.n));
        uint16_t* page = static_cast<uint16_t*>(const_cast<void*>(d.page));
        if (((reinterpret_cast<uintptr_t>(page) | reinterpret_cast<uintptr_t>(d.q)) & 15u) == 0) {
            const uint32_t v1 = e0 + (e1 - e0) / 16 * 16;
            for (uint32_t i = e0 / 16 + threadIdx.x; i < v1 / 16; i += kThreads) {
                const uint4 q = reinterpret_cast<const uint4*>(d.q)[i];
                const uint32_t in[4] = {q.x, q.y, q.z, q.w};
                uint32_t out[8];
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const uint32_t w = in[k];
                    out[2 * k] = dequantise(w & 0xffu, scale) |
                                 static_cast<uint32_t>(dequantise((w >> 8) & 0xffu, scale)) << 16;
                    out[2 * k + 1] = dequantise((w >> 16) & 0xffu, scale) |
                                     static_cast<uint32_t>(dequantise(w >> 24, scale)) << 16;
                }
                uint4* p4 = reinterpret_cast<uint4*>(page) + 2 * i;
                p4[0] = make_uint4(out[0], out[1], out[2], out[3]);
                p4[1] = make_uint4(out[4], out[5], out[6], out[7]);
            }
            for (uint32_t i = v1 + threadIdx.x; i < e1; i += kThreads) page[i] = dequantise(d.q[i], scale);
        } else {
            for (uint32_t i = e0 + threadIdx.x; i < e1; i += kThreads) page[i] = dequantise(d.q[i], scale);
        }
    }
}

__global__ void __launch_bounds__(kThreads) copy_kernel(const CopyUnit* units, uint32_t count) {
    for (uint32_t u = blockIdx.y; u < count; u += gridDim.y) {
        const CopyUnit c = units[u];
        const uint64_t begin = static_cast<uint64_t>(blockIdx.x) * kCopyChunk;
        if (begin >= c.bytes) continue;
        const uint64_t len = min(begin + kCopyChunk, c.bytes) - begin;
        const uint8_t* src = c.src + begin;
        uint8_t* dst = c.dst + begin;
        if (((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15u) == 0) {
            const uint64_t vec = len / 16;
            for (uint64_t i = threadIdx.x; i < vec; i += kThreads)
                reinterpret_cast<uint4*>(dst)[i] = __ldg(reinterpret_cast<const uint4*>(src) + i);
            for (uint64_t i = vec * 16 + threadIdx.x; i < len; i += kThreads) dst[i] = src[i];
        } else {
            for (uint64_t i = threadIdx.x; i < len; i += kThreads) dst[i] = src[i];
        }
    }
}

dim3 page_grid(uint32_t count, uint32_t max_n) {
    const uint32_t slices = (max_n + kSliceElems - 1) / kSliceElems;
    return dim3(slices ? slices : 1, count < 65535u ? count : 65535u, 1);
}

}  // namespace

cudaError_t launch_int8_encode(const Int8Unit* units, uint32_t count, uint32_t max_n,
                               cudaStream_t stream) {
    if (count == 0) return cudaSuccess;
    note_launch();
    absmax_kernel<<<page_grid(count, max_n), kThreads, 0, stream>>>(units, count);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    note_launch();
    quant_kernel<<<page_grid(count, max_n), kThreads, 0, stream>>>(units, count);
    return cudaGetLastError();
}

cudaError_t launch_int8_decode(const Int8Unit* units, uint32_t count, uint32_t max_n,
                               cudaStream_t stream) {
    if (count == 0) return cudaSuccess;
    note_launch();
    dequant_kernel<<<page_grid(count, max_n), kThreads, 0, stream>>>(units, count);
    return cudaGetLastError();
}

cudaError_t launch_copy(const CopyUnit* units, uint32_t count, uint64_t max_bytes,
                        cudaStream_t stream) {
    if (count == 0) return cudaSuccess;
    const uint64_t chunks = (max_bytes + kCopyChunk - 1) / kCopyChunk;
    dim3 grid(static_cast<uint32_t>(chunks ? chunks : 1), count < 65535u ? count : 65535u, 1);
    note_launch();
    copy_kernel<<<grid, kThreads, 0, stream>>>(units, count);
    return cudaGetLastError();
}

}  // namespace ckv
