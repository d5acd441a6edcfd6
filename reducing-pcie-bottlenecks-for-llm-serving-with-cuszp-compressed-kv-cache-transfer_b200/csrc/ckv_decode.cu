// Decoder for the fixed-mode codec (sm_100a).
//
// CTAs work on independent slices of 512 blocks (16384 elements): a slice's
// payload offset is the sum of the sizes of all earlier blocks, which the CTA
// reads straight from the unit's rate bytes (one SIMD byte-sum per four
// blocks), so no CTA waits on another and there is no global scratch.
//
//   1. offset of the slice's payload from the rate bytes before it;
//   2. one TMA bulk copy brings the slice's payload into shared memory
//      (plain word loads for the sub-16-byte tail);
//   3. per block (one per thread): sign word + planes -> register
//      transpose -> q -> (float)q * eb * 2.0f -> BF16 (round to nearest even)
//      or FP32 -> 16-byte stores to the destination of the element map
//      (contiguous page, one of several destinations, or layer-indexed
//      page).
//
// Blocks whose rate is zero are not written, as in the reference decoder
// (cuszp_batched_fixed.cu:496-623 stores only inside `if (fixed_rate)`);
// zero_fill writes (float)0 * eb * 2.0f there instead.
#include "ckv_launch.h"

namespace ckv {
namespace {

constexpr uint32_t kSliceBlocks = 512;
constexpr uint32_t kPayloadCap = kSliceBlocks * (4 + 4 * 32) + 32;
constexpr uint32_t kWaitPolls = 1u << 24;

struct DecodeArgs {
    const Unit* units;
    const Map* maps;
    uint32_t num_units;
    uint32_t zero_fill;
    uint32_t* status;
};

// Decoded values of one block, element order, from the sign word and planes.
template <bool kWide>
__device__ __forceinline__ void unpack_block(const uint32_t* words, uint32_t rate,
                                             float eb, float (&f)[32]) {
    if constexpr (!kWide) {
        // Row k holds (|q| << 1) | sign of the element at bit k, rows k and
        // k + 16 share A[k]; word 0 (the sign word) becomes bit 0 of every row.
        uint32_t A[16];
#pragma unroll
        for (int t = 0; t < 16; ++t) A[t] = t <= static_cast<int>(rate) ? words[t] : 0u;
        transpose16(A);
#pragma unroll
        for (int v = 0; v < 32; ++v) {
            const int k = bitpos(v);
            const uint32_t row = k < 16 ? (A[k] & 0xffffu) : (A[k - 16] >> 16);
            const int mag = static_cast<int>(row >> 1);
            f[v] = dequantize((row & 1u) ? -mag : mag, eb);
        }
    } else {
        uint32_t R[32];
        const uint32_t sign = words[0];
#pragma unroll
        for (int b = 0; b < 32; ++b) R[b] = b < static_cast<int>(rate) ? words[1 + b] : 0u;
        transpose32(R);
#pragma unroll
        for (int v = 0; v < 32; ++v) {
            const int k = bitpos(v);
            const int mag = static_cast<int>(R[k]);
            f[v] = dequantize(((sign >> k) & 1u) ? -mag : mag, eb);
        }
    }
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    const __nv_bfloat162 p = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&p);
}

__device__ __forceinline__ void store_elem(__nv_bfloat16* p, float v) {
    *p = __float2bfloat16_rn(v);
}
__device__ __forceinline__ void store_elem(float* p, float v) { *p = v; }

// Write the decoded block `jb` (valid elements) through the element map.
template <typename T>
__device__ __forceinline__ void write_block(const Unit& unit, const Map& map,
                                            uint32_t u, uint32_t jb,
                                            uint32_t valid, const float (&f)[32]) {
    const uint32_t e0 = jb * kBlock;
    const uint32_t L = run_len(unit, map);
    const uint32_t r0 = e0 / L, off = e0 - r0 * L;
    T* dst = run_base<T>(unit, map, u, r0) + off;
    if (valid == kBlock && off + kBlock <= L &&
        (reinterpret_cast<uintptr_t>(dst) & 15u) == 0) {
        uint4* d = reinterpret_cast<uint4*>(dst);
        if constexpr (sizeof(T) == 2) {
#pragma unroll
            for (int c = 0; c < 4; ++c)
                d[c] = make_uint4(pack_bf16x2(f[8 * c + 0], f[8 * c + 1]),
                                  pack_bf16x2(f[8 * c + 2], f[8 * c + 3]),
                                  pack_bf16x2(f[8 * c + 4], f[8 * c + 5]),
                                  pack_bf16x2(f[8 * c + 6], f[8 * c + 7]));
        } else {
#pragma unroll
            for (int c = 0; c < 8; ++c)
                d[c] = make_uint4(__float_as_uint(f[4 * c + 0]), __float_as_uint(f[4 * c + 1]),
                                  __float_as_uint(f[4 * c + 2]), __float_as_uint(f[4 * c + 3]));
        }
        return;
    }
#pragma unroll
    for (int v = 0; v < 32; ++v) {
        if (static_cast<uint32_t>(v) < valid) {
            const uint32_t i = e0 + v;
            const uint32_t r = i / L;
            store_elem(run_base<T>(unit, map, u, r) + (i - r * L), f[v]);
        }
    }
}

template <typename T>
__global__ void __launch_bounds__(kThreads) decode_kernel(DecodeArgs a) {
    extern __shared__ __align__(128) uint8_t payload[];
    __shared__ uint64_t bar;
    __shared__ uint32_t scratch[kWarps + 1];
    const int tid = threadIdx.x;
    if (tid == 0) {
        mbar_init(&bar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    uint32_t parity = 0;

    for (uint32_t u = blockIdx.y; u < a.num_units; u += gridDim.y) {
        const Unit unit = a.units[u];
        const Map map = a.maps[unit.map];
        const uint32_t n = unit.n;
        const uint32_t nb = (n + kBlock - 1) / kBlock;
        const uint32_t b0 = blockIdx.x * kSliceBlocks;
        if (b0 >= nb) continue;
        const uint32_t b1 = min(b0 + kSliceBlocks, nb);
        const uint32_t nbs = b1 - b0;
        const uint32_t hdr = (n + kGroup - 1) / kGroup * (kGroup / kBlock);
        const uint8_t* stream = unit.stream;
        const uint64_t size = unit.capacity;

        // 1. where this slice's payload starts
        uint32_t acc = 0, bad = 0, mine = 0;
        if (size >= hdr) {
            const uint32_t* words = reinterpret_cast<const uint32_t*>(stream);
            for (uint32_t w = tid; w < b0 / 4; w += kThreads) {
                const uint32_t x = __ldg(words + w);
                acc += __dp4a(x, 0x01010101u, 0u) + __dp4a(__vsetne4(x, 0u), 0x01010101u, 0u);
                bad |= __vcmpgtu4(x, 0x1f1f1f1fu);
            }
            for (uint32_t i = tid; i < nbs; i += kThreads) {
                const uint32_t r = __ldg(stream + b0 + i);
                bad |= r > 31;
                mine += r ? 4 + 4 * r : 0u;
            }
        } else {
            bad = 1;
        }
        const uint32_t prefix = 4 * cta_sum(acc, scratch);
        const uint32_t slice_total = cta_sum(mine, scratch);
        const uint64_t p0 = static_cast<uint64_t>(hdr) + prefix;
        const uint64_t p1 = p0 + slice_total;
        if (__syncthreads_or(bad != 0) || p1 > size) {
            if (tid == 0) atomicOr(&a.status[u], kErrBadStream);
            continue;
        }

        // 2. payload on chip
        const uintptr_t g0 = reinterpret_cast<uintptr_t>(stream + p0);
        const uintptr_t g1 = reinterpret_cast<uintptr_t>(stream + p1);
        const uintptr_t ga = g0 & ~uintptr_t(15), gb = g1 & ~uintptr_t(15);
        const bool bulk = gb > ga;
        if (tid == 0) {
            mbar_arrive_expect_tx(&bar, bulk ? static_cast<uint32_t>(gb - ga) : 0u);
            if (bulk)
                bulk_load(payload, reinterpret_cast<const void*>(ga),
                          static_cast<uint32_t>(gb - ga), &bar);
        }
        for (uintptr_t g = (bulk ? gb : g0) + 4 * tid; g < g1; g += 4 * kThreads)
            *reinterpret_cast<uint32_t*>(payload + (g - ga)) =
                __ldg(reinterpret_cast<const uint32_t*>(g));
        uint32_t status = 0;
        if (!mbar_wait_bounded(&bar, parity, kWaitPolls)) status |= kErrTimeout;
        parity ^= 1u;
        __syncthreads();
        const uint8_t* pay = payload + (g0 - ga);

        // 3. decode, one block per thread per round
        const float eb = unit.eb;
        uint32_t running = 0;
        const uint32_t rounds = (nbs + kThreads - 1) / kThreads;
        for (uint32_t k = 0; k < rounds; ++k) {
            const uint32_t i = k * kThreads + tid;
            const uint32_t r = i < nbs ? __ldg(stream + b0 + i) : 0u;
            uint32_t round_total;
            const uint32_t off = cta_exclusive_scan(r ? 4 + 4 * r : 0u, scratch, &round_total);
            const bool wide = __any_sync(0xffffffffu, r > 15);
            if (i < nbs && (r || a.zero_fill)) {
                const uint32_t jb = b0 + i;
                const uint32_t valid = min(n - jb * kBlock, uint32_t(kBlock));
                float f[32];
                if (r) {
                    const uint32_t* words = reinterpret_cast<const uint32_t*>(pay + running + off);
                    if (wide)
                        unpack_block<true>(words, r, eb, f);
                    else
                        unpack_block<false>(words, r, eb, f);
                } else {
                    const float z = dequantize(0, eb);
#pragma unroll
                    for (int v = 0; v < 32; ++v) f[v] = z;
                }
                write_block<T>(unit, map, u, jb, valid, f);
            }
            running += round_total;
        }
        if (status) atomicOr(&a.status[u], status);
        __syncthreads();
    }
}

template <typename T>
cudaError_t launch_decode_t(const DecodeLaunch& l, cudaStream_t stream) {
    if (l.num_units == 0) return cudaErrorInvalidValue;
    const uint32_t nb_max = (l.max_n + kBlock - 1) / kBlock;
    const uint32_t slices = (nb_max + kSliceBlocks - 1) / kSliceBlocks;
    auto kernel = decode_kernel<T>;
    cudaError_t err = cudaFuncSetAttribute(
        kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kPayloadCap);
    if (err != cudaSuccess) return err;
    DecodeArgs args{l.units, l.maps, l.num_units, l.zero_fill ? 1u : 0u, l.status};
    dim3 grid(slices ? slices : 1, l.num_units < 65535u ? l.num_units : 65535u, 1);
    note_launch();
    decode_kernel<T><<<grid, kThreads, kPayloadCap, stream>>>(args);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_decode(const DecodeLaunch& l, cudaStream_t stream) {
    if (l.type == ElemType::kBF16) return launch_decode_t<__nv_bfloat16>(l, stream);
    return launch_decode_t<float>(l, stream);
}

}  // namespace ckv
