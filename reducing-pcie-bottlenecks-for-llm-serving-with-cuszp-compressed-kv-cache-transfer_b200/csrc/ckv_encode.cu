// Single-pass clustered encoder for the fixed-mode codec (sm_100a).
//
// One thread-block cluster encodes one unit (a KV page, or the selected
// layers of one).  Each CTA of the cluster owns a contiguous slice of the
// unit's 32-element blocks and keeps that slice in shared memory for the
// whole encode, so HBM is read once and written once:
//
//   1. TMA bulk copies bring the slice into shared memory (one copy per
//      contiguous run of the element map);
//   2. per block, min / max / NaN-presence (packed BF16 min/max);
//   3. the CTAs exchange their slice extremes through distributed shared
//      memory -> every CTA resolves the same absolute bound
//      eb = eps * fmaxf(max - min, 1e-6f) (cuszp_batched_fixed.cu:55-133);
//   4. per block rate = bit length of max(|q(block min)|, |q(block max)|)
//      -- the quantiser is monotone, so the extremes give the block's
//      largest |q| (NaN contributes |q| = 1) -- then the CTAs exchange
//      their slice byte totals -> each CTA knows where its output starts;
//      no look-back chain, no global scratch;
//   5. per block: quantise the 32 values, transpose them into the sign word
//      and bit planes in registers, stage the round's output in shared
//      memory and write it back with a TMA bulk store (plain stores for the
//      unaligned head and tail words).
//
// The rate found in step 5 from the values themselves is checked against
// the one from step 4; a mismatch sets kErrRateCheck.
#include "ckv_launch.h"

#include <cooperative_groups.h>

#include <cfloat>

namespace cg = cooperative_groups;

namespace ckv {
namespace {

constexpr uint32_t kSliceBytes = 64 * 1024;
constexpr uint32_t kStageCap = 16384 + 16;
constexpr uint32_t kMaxCluster = 16;
constexpr uint32_t kWaitPolls = 1u << 24;
constexpr uint32_t kMaxPieces = 512;

template <typename T>
struct Traits;
template <>
struct Traits<__nv_bfloat16> {
    static constexpr uint32_t kBytes = 2;
};
template <>
struct Traits<float> {
    static constexpr uint32_t kBytes = 4;
};

template <typename T>
struct Layout {
    static constexpr uint32_t kBlocks = kSliceBytes / (kBlock * Traits<T>::kBytes);
    static constexpr uint32_t kSlice = 0;
    static constexpr uint32_t kMinMax = kSliceBytes;
    static constexpr uint32_t kRates = kMinMax + kBlocks * 8;
    static constexpr uint32_t kStageStride = (kStageCap + 15) / 16 * 16;
    static constexpr uint32_t kStage = kRates + (kBlocks + 15) / 16 * 16;
    static constexpr uint32_t kTotal = kStage + 2 * kStageStride;
};

struct EncodeArgs {
    const Unit* units;
    const Map* maps;
    uint32_t num_units;
    uint32_t relative;
    uint64_t* sizes;
    float* bounds;
    uint32_t* status;
};

// Thread 0: plan the slice load [e0, e1) as bulk copies of 16-byte aligned
// runs.  Returns false when some run cannot be bulk-copied (then every
// element is copied by the threads).  *tail is the first element of the
// sub-16-byte tail that the threads copy.
template <typename T>
__device__ bool plan_and_issue_load(const Unit& unit, const Map& m, uint32_t u,
                                    uint32_t e0, uint32_t e1, uint8_t* slice,
                                    uint64_t* bar, uint32_t* tail) {
    constexpr uint32_t B = Traits<T>::kBytes;
    const uint32_t L = run_len(unit, m);
    uint32_t total = 0, pieces = 0;
    *tail = e1;
    bool ok = true;
    for (uint32_t pos = e0; pos < e1;) {
        const uint32_t r = pos / L, off = pos - r * L;
        const uint32_t len = min(e1 - pos, L - off);
        const T* src = run_base<const T>(unit, m, u, r) + off;
        const uint32_t bytes = len * B, body = bytes & ~15u;
        const bool last = pos + len == e1;
        if ((reinterpret_cast<uintptr_t>(src) & 15u) || (((pos - e0) * B) & 15u) ||
            (!last && body != bytes) || ++pieces > kMaxPieces) {
            ok = false;
            break;
        }
        total += body;
        if (last) *tail = pos + body / B;
        pos += len;
    }
    if (!ok) {
        *tail = e0;
        mbar_arrive_expect_tx(bar, 0);
        return false;
    }
    mbar_arrive_expect_tx(bar, total);
    for (uint32_t pos = e0; pos < e1;) {
        const uint32_t r = pos / L, off = pos - r * L;
        const uint32_t len = min(e1 - pos, L - off);
        const T* src = run_base<const T>(unit, m, u, r) + off;
        const uint32_t body = (len * B) & ~15u;
        if (body) bulk_load(slice + (pos - e0) * B, src, body, bar);
        pos += len;
    }
    return true;
}

template <typename T>
__device__ void copy_elements(const Unit& unit, const Map& m, uint32_t u,
                              uint32_t from, uint32_t to, uint32_t e0,
                              uint8_t* slice) {
    const uint32_t L = run_len(unit, m);
    T* dst = reinterpret_cast<T*>(slice);
    for (uint32_t i = from + threadIdx.x; i < to; i += kThreads) {
        const uint32_t r = i / L;
        dst[i - e0] = run_base<const T>(unit, m, u, r)[i - r * L];
    }
}

// ---- per-block extremes ---------------------------------------------------

// rho rotates which 16-byte chunk a thread reads first, so that the eight
// threads of a shared-memory phase hit eight different bank groups.
__device__ __forceinline__ void block_extremes(const uint8_t* blk, int rho,
                                               float& lo, float& hi, bool& nan,
                                               __nv_bfloat16) {
    const uint4* p = reinterpret_cast<const uint4*>(blk);
    __nv_bfloat162 w[16];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint4 c = p[(j + rho) & 3];
        w[4 * j + 0] = *reinterpret_cast<const __nv_bfloat162*>(&c.x);
        w[4 * j + 1] = *reinterpret_cast<const __nv_bfloat162*>(&c.y);
        w[4 * j + 2] = *reinterpret_cast<const __nv_bfloat162*>(&c.z);
        w[4 * j + 3] = *reinterpret_cast<const __nv_bfloat162*>(&c.w);
    }
    __nv_bfloat162 mn[8], mx[8], mz[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        mn[k] = __hmin2(w[2 * k], w[2 * k + 1]);
        mx[k] = __hmax2(w[2 * k], w[2 * k + 1]);
        mz[k] = __hmax2_nan(w[2 * k], w[2 * k + 1]);
    }
#pragma unroll
    for (int s = 4; s >= 1; s >>= 1) {
#pragma unroll
        for (int k = 0; k < s; ++k) {
            mn[k] = __hmin2(mn[k], mn[k + s]);
            mx[k] = __hmax2(mx[k], mx[k + s]);
            mz[k] = __hmax2_nan(mz[k], mz[k + s]);
        }
    }
    lo = fminf(__low2float(mn[0]), __high2float(mn[0]));
    hi = fmaxf(__low2float(mx[0]), __high2float(mx[0]));
    const float a = __low2float(mz[0]), b = __high2float(mz[0]);
    nan = (a != a) || (b != b);
}

__device__ __forceinline__ float nanmax(float a, float b) {
    float r;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    return r;
}

__device__ __forceinline__ void block_extremes(const uint8_t* blk, int rho,
                                               float& lo, float& hi, bool& nan,
                                               float) {
    const uint4* p = reinterpret_cast<const uint4*>(blk);
    float x[32];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int c = (j + rho) & 3;
        const uint4 a = p[2 * c], b = p[2 * c + 1];
        x[8 * j + 0] = __uint_as_float(a.x);
        x[8 * j + 1] = __uint_as_float(a.y);
        x[8 * j + 2] = __uint_as_float(a.z);
        x[8 * j + 3] = __uint_as_float(a.w);
        x[8 * j + 4] = __uint_as_float(b.x);
        x[8 * j + 5] = __uint_as_float(b.y);
        x[8 * j + 6] = __uint_as_float(b.z);
        x[8 * j + 7] = __uint_as_float(b.w);
    }
    float mn[16], mx[16], mz[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) {
        mn[k] = fminf(x[2 * k], x[2 * k + 1]);
        mx[k] = fmaxf(x[2 * k], x[2 * k + 1]);
        mz[k] = nanmax(x[2 * k], x[2 * k + 1]);
    }
#pragma unroll
    for (int s = 8; s >= 1; s >>= 1) {
#pragma unroll
        for (int k = 0; k < s; ++k) {
            mn[k] = fminf(mn[k], mn[k + s]);
            mx[k] = fmaxf(mx[k], mx[k + s]);
            mz[k] = nanmax(mz[k], mz[k + s]);
        }
    }
    lo = mn[0];
    hi = mx[0];
    nan = mz[0] != mz[0];
}

template <typename T>
__device__ __forceinline__ float elem_value(const uint8_t* blk, int v) {
    if constexpr (sizeof(T) == 2) {
        const uint16_t b = reinterpret_cast<const uint16_t*>(blk)[v];
        return __uint_as_float(static_cast<uint32_t>(b) << 16);
    } else {
        return reinterpret_cast<const float*>(blk)[v];
    }
}

// ---- packing --------------------------------------------------------------

// Quantised values of one block in register order e = 8*j + u, where
// register byte lane j holds block byte lane (j + rho) & 3.
template <typename T>
__device__ __forceinline__ void quantise_block(const uint8_t* blk, int rho,
                                               float recip, uint32_t valid,
                                               int (&q)[32]) {
    if constexpr (sizeof(T) == 2) {
        const uint4* p = reinterpret_cast<const uint4*>(blk);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint4 c = p[(j + rho) & 3];
            const uint32_t w[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
            for (int m = 0; m < 4; ++m) {
                q[8 * j + 2 * m] = quantize(bf16_lo(w[m]), recip);
                q[8 * j + 2 * m + 1] = quantize(bf16_hi(w[m]), recip);
            }
        }
    } else {
        const uint4* p = reinterpret_cast<const uint4*>(blk);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int c = (j + rho) & 3;
            const uint4 a = p[2 * c], b = p[2 * c + 1];
            const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
            for (int m = 0; m < 8; ++m)
                q[8 * j + m] = quantize(__uint_as_float(w[m]), recip);
        }
    }
    if (valid < 32) {
        // Elements past the end of the unit count as zero
        // (cuszp_batched_fixed.cu:200-211).
#pragma unroll
        for (int e = 0; e < 32; ++e) {
            const uint32_t v = 8u * (((e >> 3) + rho) & 3) + (e & 7);
            if (v >= valid) q[e] = 0;
        }
    }
}

__device__ __forceinline__ uint32_t signed_row(int q) {
    // (|q| << 1) | sign: bit 0 of every row becomes the sign word.
    return (uabs(q) << 1) | (static_cast<uint32_t>(q) >> 31);
}

// Writes the sign word and `rate` planes of one block to out[0..rate].
template <bool kWide>
__device__ __forceinline__ void emit_block(const int (&q)[32], int rho,
                                           uint32_t rate, uint32_t* out) {
    const uint32_t sh = 8u * rho;
    if constexpr (!kWide) {
        uint32_t A[16];
#pragma unroll
        for (int k = 0; k < 16; ++k) {
            const int e = bitpos(k);
            A[k] = signed_row(q[e]) | (signed_row(q[e + 16]) << 16);
        }
        transpose16(A);
#pragma unroll
        for (int t = 0; t < 16; ++t)
            if (t <= static_cast<int>(rate)) out[t] = __funnelshift_l(A[t], A[t], sh);
    } else {
        uint32_t R[32];
        uint32_t sign = 0;
#pragma unroll
        for (int k = 0; k < 32; ++k) {
            const int e = bitpos(k);
            R[k] = uabs(q[e]);
            sign |= (static_cast<uint32_t>(q[e]) >> 31) << k;
        }
        transpose32(R);
        out[0] = __funnelshift_l(sign, sign, sh);
#pragma unroll
        for (int b = 0; b < 32; ++b)
            if (b < static_cast<int>(rate)) out[1 + b] = __funnelshift_l(R[b], R[b], sh);
    }
}

// ---- the kernel -------------------------------------------------------------

template <typename T>
__global__ void __launch_bounds__(kThreads, 2) encode_kernel(EncodeArgs a) {
    using L = Layout<T>;
    constexpr uint32_t B = Traits<T>::kBytes;
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t* slice = smem + L::kSlice;
    float2* extremes = reinterpret_cast<float2*>(smem + L::kMinMax);
    uint8_t* rates = smem + L::kRates;
    uint8_t* stage0 = smem + L::kStage;

    __shared__ uint64_t bar;
    __shared__ uint32_t scratch[kWarps + 1];
    __shared__ float red_lo[kWarps], red_hi[kWarps];
    __shared__ float2 s_extremes;     // read by the other CTAs of the cluster
    __shared__ uint32_t s_total;      // read by the other CTAs of the cluster
    __shared__ uint32_t s_base, s_unit_total, s_tail, s_bulk_ok, s_status;
    __shared__ float s_eb;

    cg::cluster_group cluster = cg::this_cluster();
    const uint32_t rank = cluster.block_rank();
    const uint32_t csize = cluster.num_blocks();
    const int tid = threadIdx.x;
    const int rho = (sizeof(T) == 2) ? ((tid >> 1) & 3) : (tid & 3);

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
        const uint32_t sb = (nb + csize - 1) / csize;
        const uint32_t b0 = min(rank * sb, nb), b1 = min(b0 + sb, nb);
        const uint32_t nbs = b1 - b0;
        const uint32_t e0 = b0 * kBlock, e1 = min(b1 * kBlock, n);
        const uint32_t hdr = (n + kGroup - 1) / kGroup * (kGroup / kBlock);
        uint32_t status = 0;

        // 1. bring the slice on chip
        if (tid == 0) {
            s_status = 0;
            uint32_t tail;
            s_bulk_ok = plan_and_issue_load<T>(unit, map, u, e0, e1, slice, &bar, &tail);
            s_tail = tail;
        }
        __syncthreads();
        copy_elements<T>(unit, map, u, s_tail, e1, e0, slice);
        if (!mbar_wait_bounded(&bar, parity, kWaitPolls)) status |= kErrTimeout;
        parity ^= 1u;
        __syncthreads();

        // 2. block extremes
        float tlo = FLT_MAX, thi = -FLT_MAX;
        for (uint32_t i = tid; i < nbs; i += kThreads) {
            const uint8_t* blk = slice + i * kBlock * B;
            float lo, hi;
            bool nan;
            const uint32_t valid = min(n - (b0 + i) * kBlock, uint32_t(kBlock));
            if (valid == kBlock) {
                block_extremes(blk, rho, lo, hi, nan, T());
            } else {
                lo = __int_as_float(0x7fffffff);
                hi = lo;
                nan = false;
                for (uint32_t v = 0; v < valid; ++v) {
                    const float x = elem_value<T>(blk, v);
                    lo = fminf(lo, x);
                    hi = fmaxf(hi, x);
                    nan |= x != x;
                }
            }
            extremes[i] = make_float2(lo, hi);
            rates[i] = nan ? 1 : 0;
            tlo = fminf(tlo, lo);
            thi = fmaxf(thi, hi);
        }
#pragma unroll
        for (int d = 16; d > 0; d >>= 1) {
            tlo = fminf(tlo, __shfl_xor_sync(0xffffffffu, tlo, d));
            thi = fmaxf(thi, __shfl_xor_sync(0xffffffffu, thi, d));
        }
        if ((tid & 31) == 0) {
            red_lo[tid >> 5] = tlo;
            red_hi[tid >> 5] = thi;
        }
        __syncthreads();
        if (tid == 0) {
            float lo = FLT_MAX, hi = -FLT_MAX;
#pragma unroll
            for (int w = 0; w < kWarps; ++w) {
                lo = fminf(lo, red_lo[w]);
                hi = fmaxf(hi, red_hi[w]);
            }
            s_extremes = make_float2(lo, hi);
        }

        // 3. unit extremes through distributed shared memory -> bound
        cluster.sync();
        if (tid == 0) {
            float lo = FLT_MAX, hi = -FLT_MAX;
            for (uint32_t r = 0; r < csize; ++r) {
                const float2 v = *cluster.map_shared_rank(&s_extremes, r);
                lo = fminf(lo, v.x);
                hi = fmaxf(hi, v.y);
            }
            s_eb = resolve_bound(unit.eb, lo, hi, a.relative != 0);
        }
        __syncthreads();
        const float eb = s_eb;
        const float recip = __fdiv_rn(0.5f, eb);

        // 4. rates and slice size, then slice offsets across the cluster
        uint32_t mine = 0;
        for (uint32_t i = tid; i < nbs; i += kThreads) {
            const float2 mm = extremes[i];
            uint32_t m = 0;
            if (mm.x == mm.x)
                m = max(uabs(quantize(mm.x, recip)), uabs(quantize(mm.y, recip)));
            if (rates[i]) m = max(m, 1u);
            const uint32_t r = 32 - __clz(m);
            rates[i] = static_cast<uint8_t>(r);
            mine += r ? 4 + 4 * r : 0;
        }
        const uint32_t slice_total = cta_sum(mine, scratch);
        if (tid == 0) s_total = slice_total;
        cluster.sync();
        if (tid == 0) {
            uint32_t base = 0, all = 0;
            for (uint32_t r = 0; r < csize; ++r) {
                const uint32_t t = *cluster.map_shared_rank(&s_total, r);
                base += r < rank ? t : 0u;
                all += t;
            }
            s_base = base;
            s_unit_total = all;
        }
        auto done_reading = cluster.barrier_arrive();
        __syncthreads();
        const uint64_t unit_bytes = static_cast<uint64_t>(hdr) + s_unit_total;
        const bool fits = unit_bytes <= unit.capacity;
        if (rank == 0 && tid == 0) {
            a.sizes[u] = unit_bytes;
            a.bounds[u] = eb;
        }
        if (!fits) status |= kErrCapacity;

        if (fits) {
            uint8_t* stream = unit.stream;
            // rate bytes of this slice; the last CTA zeroes the unused ones
            for (uint32_t i = tid; i < nbs; i += kThreads) stream[b0 + i] = rates[i];
            if (rank == csize - 1)
                for (uint32_t j = nb + tid; j < hdr; j += kThreads) stream[j] = 0;

            // 5. pack, round by round (one block per thread per round)
            uint32_t running = hdr + s_base;
            const uint32_t rounds = (nbs + kThreads - 1) / kThreads;
            for (uint32_t k = 0; k < rounds; ++k) {
                if (tid == 0 && k >= 2) bulk_wait_read<1>();
                const uint32_t i = k * kThreads + tid;
                const uint32_t r = i < nbs ? rates[i] : 0u;
                uint32_t round_total;
                const uint32_t off = cta_exclusive_scan(r ? 4 + 4 * r : 0u, scratch, &round_total);
                const uint32_t start = running;
                const uint32_t shift = start & 15u;
                uint8_t* stage = stage0 + (k & 1) * L::kStageStride;
                const bool staged = shift + round_total <= kStageCap;
                uint32_t* out = reinterpret_cast<uint32_t*>(
                    staged ? stage + shift + off : stream + start + off);
                const bool wide = __any_sync(0xffffffffu, r > 15);
                if (r) {
                    int q[32];
                    const uint32_t valid = min(n - (b0 + i) * kBlock, uint32_t(kBlock));
                    quantise_block<T>(slice + i * kBlock * B, rho, recip, valid, q);
                    uint32_t orv = 0;
#pragma unroll
                    for (int e = 0; e < 32; ++e) orv |= uabs(q[e]);
                    if (32u - __clz(orv) != r) status |= kErrRateCheck;
                    if (wide)
                        emit_block<true>(q, rho, r, out);
                    else
                        emit_block<false>(q, rho, r, out);
                } else if (i < nbs) {
                    // A rate-0 block must really be all zeros.
                    int q[32];
                    const uint32_t valid = min(n - (b0 + i) * kBlock, uint32_t(kBlock));
                    quantise_block<T>(slice + i * kBlock * B, rho, recip, valid, q);
                    uint32_t orv = 0;
#pragma unroll
                    for (int e = 0; e < 32; ++e) orv |= uabs(q[e]);
                    if (orv) status |= kErrRateCheck;
                }
                if (staged) {
                    fence_proxy_async_smem();
                    __syncthreads();
                    const uint32_t end = start + round_total;
                    const uint32_t a0 = (start + 15u) & ~15u, a1 = end & ~15u;
                    const bool body = a1 > a0;
                    const uint32_t head_end = body ? a0 : end;
                    if (body && tid == 0) {
                        bulk_store(stream + a0, stage + shift + (a0 - start), a1 - a0);
                        bulk_commit();
                    }
                    const uint32_t head_words = (head_end - start) >> 2;
                    const uint32_t tail_words = body ? (end - a1) >> 2 : 0u;
                    if (tid < head_words) {
                        reinterpret_cast<uint32_t*>(stream + start)[tid] =
                            reinterpret_cast<const uint32_t*>(stage + shift)[tid];
                    } else if (tid >= 32 && tid - 32 < tail_words) {
                        const uint32_t t = tid - 32;
                        reinterpret_cast<uint32_t*>(stream + a1)[t] =
                            reinterpret_cast<const uint32_t*>(stage + shift + (a1 - start))[t];
                    }
                } else {
                    __syncthreads();
                }
                running += round_total;
            }
            if (tid == 0) bulk_wait<0>();
        }
        if (status) atomicOr(&s_status, status);
        __syncthreads();
        // Status lives in mapped host memory: a plain store (no atomics over
        // PCIe); any CTA that saw an error leaves a nonzero word.
        if (tid == 0 && s_status)
            *reinterpret_cast<volatile uint32_t*>(&a.status[u]) = s_status;
        cluster.barrier_wait(std::move(done_reading));
    }
}

template <typename T>
cudaError_t launch_encode_t(const EncodeLaunch& l, cudaStream_t stream) {
    using L = Layout<T>;
    const uint32_t nb_max = (l.max_n + kBlock - 1) / kBlock;
    uint32_t c = (nb_max + L::kBlocks - 1) / L::kBlocks;
    if (c == 0) c = 1;
    if (c > kMaxCluster || l.num_units == 0) return cudaErrorInvalidValue;
    auto kernel = encode_kernel<T>;
    cudaError_t err = cudaFuncSetAttribute(
        kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kTotal);
    if (err != cudaSuccess) return err;
    if (c > 8) {
        err = cudaFuncSetAttribute(kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        if (err != cudaSuccess) return err;
    }
    EncodeArgs args{l.units, l.maps, l.num_units, l.relative ? 1u : 0u,
                    l.sizes, l.bounds, l.status};
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(c, l.num_units < 65535u ? l.num_units : 65535u, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = L::kTotal;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = c;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    note_launch();
    return cudaLaunchKernelEx(&cfg, kernel, args);
}

}  // namespace

uint32_t encode_max_elements(ElemType type) {
    return type == ElemType::kBF16 ? kMaxCluster * Layout<__nv_bfloat16>::kBlocks * kBlock
                                   : kMaxCluster * Layout<float>::kBlocks * kBlock;
}

cudaError_t launch_encode(const EncodeLaunch& l, cudaStream_t stream) {
    if (l.type == ElemType::kBF16) return launch_encode_t<__nv_bfloat16>(l, stream);
    return launch_encode_t<float>(l, stream);
}

}  // namespace ckv
