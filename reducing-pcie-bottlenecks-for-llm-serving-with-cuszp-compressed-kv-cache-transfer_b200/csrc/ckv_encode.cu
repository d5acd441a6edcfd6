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
//      memory (each CTA stores into every peer before a cluster barrier and
//      reads locally after it) -> every CTA resolves the same absolute bound
//      eb = eps * fmaxf(max - min, 1e-6f) (cuszp_batched_fixed.cu:55-133);
//   4. per block rate = bit length of max(|q(block min)|, |q(block max)|)
//      -- the quantiser is monotone, so the extremes give the block's
//      largest |q| (NaN contributes |q| = 1) -- one CTA scan gives every
//      block's payload offset, and the CTAs exchange their slice byte totals
//      -> each CTA knows where its output starts; no look-back chain, no
//      global scratch;
//   5. per round of 256 blocks (one per thread): quantise the 32 values,
//      transpose them into the sign word and bit planes in registers, and
//      write them IN PLACE over the already consumed input in shared memory
//      (a block of rate <= 15 packs into at most the 64 bytes it came from);
//      at the end one TMA bulk store writes the slice's payload.
//
// Rate <= 15 blocks without NaN (every block at REL bounds >= 1e-5 on
// two-sided data) use a quantiser that truncates with a round-toward-zero
// add of 2^23 instead of a float->int conversion; it gives the reference's
// integer for |q| < 2^15.  Other blocks use the reference's exact
// instruction sequence and are written straight to global memory.
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
constexpr uint32_t kGuard = 16;     // in-place output may start up to 15 bytes early
constexpr uint32_t kMaxCluster = 16;
constexpr uint32_t kWaitPolls = 1u << 24;
constexpr uint32_t kMaxPieces = 512;
constexpr uint8_t kNanFlag = 0x80;

template <typename T>
struct Traits;
template <>
struct Traits<__nv_bfloat16> {
    static constexpr uint32_t kBytes = 2;
    static constexpr int kWords = 16;   // 32-bit words per block
};
template <>
struct Traits<float> {
    static constexpr uint32_t kBytes = 4;
    static constexpr int kWords = 32;
};

template <typename T>
struct Layout {
    static constexpr uint32_t kBlocks = kSliceBytes / (kBlock * Traits<T>::kBytes);
    static constexpr uint32_t kRounds = kBlocks / kThreads;
    static constexpr uint32_t kSlice = kGuard;
    static constexpr uint32_t kExtremes = kGuard + kSliceBytes;   // 4 KB either type
    static constexpr uint32_t kRates = kExtremes + 4096;
    static constexpr uint32_t kTotal = kRates + (kBlocks + 15) / 16 * 16;
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

// ---- slice load ------------------------------------------------------------

// Thread 0: plan the slice load [e0, e1) as bulk copies of 16-byte aligned
// runs.  Returns false when some run cannot be bulk-copied (then every
// element is copied by the threads).  *tail is the first element of the
// sub-16-byte tail that the threads copy.
template <typename T>
__device__ bool plan_and_issue_load(const Unit& unit, const Map& m, uint32_t u, uint32_t e0,
                                    uint32_t e1, uint8_t* slice, uint64_t* bar, uint32_t* tail) {
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
__device__ void copy_elements(const Unit& unit, const Map& m, uint32_t u, uint32_t from,
                              uint32_t to, uint32_t e0, uint8_t* slice) {
    const uint32_t L = run_len(unit, m);
    T* dst = reinterpret_cast<T*>(slice);
    for (uint32_t i = from + threadIdx.x; i < to; i += kThreads) {
        const uint32_t r = i / L;
        dst[i - e0] = run_base<const T>(unit, m, u, r)[i - r * L];
    }
}

// ---- one block in registers ------------------------------------------------

// The words of one block.  rho rotates which 8-element byte lane a thread
// reads first, so that the eight threads of a shared-memory phase hit eight
// different bank groups; register element e = 8*j + u holds block element
// 8*((j + rho) & 3) + u.
template <typename T>
__device__ __forceinline__ void load_block(const uint8_t* blk, int rho,
                                           uint32_t (&w)[Traits<T>::kWords]) {
    const uint4* p = reinterpret_cast<const uint4*>(blk);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int c = (j + rho) & 3;
        if constexpr (sizeof(T) == 2) {
            const uint4 a = p[c];
            w[4 * j + 0] = a.x;
            w[4 * j + 1] = a.y;
            w[4 * j + 2] = a.z;
            w[4 * j + 3] = a.w;
        } else {
            const uint4 a = p[2 * c], b = p[2 * c + 1];
            w[8 * j + 0] = a.x;
            w[8 * j + 1] = a.y;
            w[8 * j + 2] = a.z;
            w[8 * j + 3] = a.w;
            w[8 * j + 4] = b.x;
            w[8 * j + 5] = b.y;
            w[8 * j + 6] = b.z;
            w[8 * j + 7] = b.w;
        }
    }
}

template <typename T>
__device__ __forceinline__ float elem(const uint32_t (&w)[Traits<T>::kWords], int e) {
    if constexpr (sizeof(T) == 2)
        return (e & 1) ? bf16_hi(w[e >> 1]) : bf16_lo(w[e >> 1]);
    else
        return __uint_as_float(w[e]);
}

__device__ __forceinline__ bool masked(int e, int rho, uint32_t valid) {
    return static_cast<uint32_t>(8 * (((e >> 3) + rho) & 3) + (e & 7)) >= valid;
}

// (|q| << 1) | sign for |q| < 2^15 and no NaN: truncation by a
// round-toward-zero add of 2^23 (exact for |t| < 2^23), the rest as
// batch_quantization (cuszp_batched_fixed.cu:10-25).
__device__ __forceinline__ uint32_t narrow_row(float x, float recip) {
    const float r = __fmul_rn(x, recip);
    const float t = __fadd_rn(r, 0.5f);
    const float z = __fadd_rz(fabsf(t), 8388608.0f);
    const uint32_t twice = (__float_as_uint(z) << 1) - 0x96000000u;  // 2 * trunc(|t|)
    return r >= -0.5f ? twice : twice + 3u;  // |q| = trunc(|t|) + s, sign = s
}

// Rows of the 16x32 bit matrix for a narrow block: A[k] holds rows k and
// k + 16, then the transpose turns them into the sign word (A[0]) and the
// planes (A[1 + b]).  Elements past the end of the unit were set to +0 in
// shared memory, which quantises to 0 for a finite 0.5 / eb.  Returns the
// OR of all rows.
template <typename T>
__device__ __forceinline__ uint32_t narrow_block(const uint32_t (&w)[Traits<T>::kWords],
                                                 float recip, uint32_t (&A)[16]) {
    uint32_t orv = 0;
#pragma unroll
    for (int k = 0; k < 16; ++k) {
        const int e = bitpos(k);
        const uint32_t lo = narrow_row(elem<T>(w, e), recip);
        const uint32_t hi = narrow_row(elem<T>(w, e + 16), recip);
        orv |= lo | hi;
        A[k] = __byte_perm(lo, hi, 0x5410);
    }
    transpose16(A);
    return orv;
}

// Exact quantiser (the reference's instruction sequence) for one element.
template <typename T>
__device__ __forceinline__ int exact_q(const uint32_t (&w)[Traits<T>::kWords], int e, int rho,
                                       float recip, uint32_t valid) {
    if (valid < kBlock && masked(e, rho, valid)) return 0;
    return quantize(elem<T>(w, e), recip);
}

// Any block: sign word and `rate` planes to out[0..rate] (nothing for rate
// 0), two 16-row transposes (low and high halves of |q|).  Returns the OR
// of |q|.
template <typename T>
__device__ __forceinline__ uint32_t wide_block(const uint32_t (&w)[Traits<T>::kWords], int rho,
                                               float recip, uint32_t valid, uint32_t rate,
                                               uint32_t* out) {
    const uint32_t sh = 8u * rho;
    uint32_t sign = 0, orv = 0;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
        uint32_t A[16];
#pragma unroll
        for (int k = 0; k < 16; ++k) {
            const int e = bitpos(k);
            const int q1 = exact_q<T>(w, e, rho, recip, valid);
            const int q2 = exact_q<T>(w, e + 16, rho, recip, valid);
            const uint32_t a1 = uabs(q1), a2 = uabs(q2);
            if (half == 0) {
                sign |= (static_cast<uint32_t>(q1) >> 31) << k;
                sign |= (static_cast<uint32_t>(q2) >> 31) << (k + 16);
                orv |= a1 | a2;
                A[k] = __byte_perm(a1, a2, 0x5410);
            } else {
                A[k] = __byte_perm(a1, a2, 0x7632);
            }
        }
        transpose16(A);
#pragma unroll
        for (int b = 0; b < 16; ++b)
            if (16 * half + b < static_cast<int>(rate))
                out[1 + 16 * half + b] = __funnelshift_l(A[b], A[b], sh);
    }
    if (rate) out[0] = __funnelshift_l(sign, sign, sh);
    return orv;
}

template <typename T>
__device__ __forceinline__ void block_extremes(const uint32_t (&w)[Traits<T>::kWords], float& lo,
                                               float& hi, bool& nan);

template <>
__device__ __forceinline__ void block_extremes<__nv_bfloat16>(const uint32_t (&w)[16], float& lo,
                                                              float& hi, bool& nan) {
    __nv_bfloat162 mn[8], mx[8], mz[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(&w[2 * k]);
        const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&w[2 * k + 1]);
        mn[k] = __hmin2(a, b);
        mx[k] = __hmax2(a, b);
        mz[k] = __hmax2_nan(a, b);
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

template <>
__device__ __forceinline__ void block_extremes<float>(const uint32_t (&w)[32], float& lo,
                                                      float& hi, bool& nan) {
    float mn[16], mx[16], mz[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) {
        const float a = __uint_as_float(w[2 * k]), b = __uint_as_float(w[2 * k + 1]);
        mn[k] = fminf(a, b);
        mx[k] = fmaxf(a, b);
        mz[k] = nanmax(a, b);
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
__device__ __forceinline__ float elem_at(const uint8_t* blk, int v) {
    if constexpr (sizeof(T) == 2)
        return __uint_as_float(static_cast<uint32_t>(reinterpret_cast<const uint16_t*>(blk)[v]) << 16);
    else
        return reinterpret_cast<const float*>(blk)[v];
}

// ---- the kernel --------------------------------------------------------------

template <typename T>
__global__ void __launch_bounds__(kThreads, 3) encode_kernel(EncodeArgs a) {
    using L = Layout<T>;
    constexpr uint32_t BB = kBlock * Traits<T>::kBytes;  // input bytes per block
    constexpr int R = static_cast<int>(L::kRounds);
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t* slice = smem + L::kSlice;
    float2* ext32 = reinterpret_cast<float2*>(smem + L::kExtremes);
    uint32_t* ext16 = reinterpret_cast<uint32_t*>(smem + L::kExtremes);
    uint8_t* rates = smem + L::kRates;
    uint32_t* offs = reinterpret_cast<uint32_t*>(smem + L::kExtremes);  // after phase 4

    __shared__ uint64_t bar;
    __shared__ uint32_t wsum[R][kWarps];
    __shared__ float red_lo[kWarps], red_hi[kWarps];
    // Written by every CTA of the cluster into every CTA (distributed shared
    // memory stores before a cluster barrier), read locally after it.
    __shared__ float2 s_extremes[kMaxCluster];
    __shared__ uint32_t s_totals[kMaxCluster];
    __shared__ uint32_t s_base, s_unit_total, s_tail, s_status;
    __shared__ float s_eb, s_recip;

    cg::cluster_group cluster = cg::this_cluster();
    const uint32_t rank = cluster.block_rank();
    const uint32_t csize = cluster.num_blocks();
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
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

        // 1. the slice on chip
        if (tid == 0) {
            s_status = 0;
            uint32_t tail;
            plan_and_issue_load<T>(unit, map, u, e0, e1, slice, &bar, &tail);
            s_tail = tail;
        }
        __syncthreads();
        copy_elements<T>(unit, map, u, s_tail, e1, e0, slice);
        if (!mbar_wait_bounded(&bar, parity, kWaitPolls)) status |= kErrTimeout;
        parity ^= 1u;
        // +0 past the end of the unit (the last block may be partial)
        if (b1 == nb && nbs && tid < static_cast<int>(b1 * kBlock - e1))
            reinterpret_cast<T*>(slice)[e1 - e0 + tid] = T(0.0f);
        __syncthreads();

        // 2. block extremes
        float tlo = FLT_MAX, thi = -FLT_MAX;
        for (uint32_t i = tid; i < nbs; i += kThreads) {
            const uint8_t* blk = slice + i * BB;
            float lo, hi;
            bool nan;
            const uint32_t valid = min(n - (b0 + i) * kBlock, uint32_t(kBlock));
            if (valid == kBlock) {
                uint32_t w[Traits<T>::kWords];
                load_block<T>(blk, rho, w);
                block_extremes<T>(w, lo, hi, nan);
            } else {
                lo = __int_as_float(0x7fffffff);
                hi = lo;
                nan = false;
                for (uint32_t v = 0; v < valid; ++v) {
                    const float x = elem_at<T>(blk, v);
                    lo = fminf(lo, x);
                    hi = fmaxf(hi, x);
                    nan |= x != x;
                }
            }
            if constexpr (sizeof(T) == 2)
                ext16[i] = (__float_as_uint(lo) >> 16) | (__float_as_uint(hi) & 0xffff0000u);
            else
                ext32[i] = make_float2(lo, hi);
            rates[i] = nan ? kNanFlag : 0;
            tlo = fminf(tlo, lo);
            thi = fmaxf(thi, hi);
        }
#pragma unroll
        for (int d = 16; d > 0; d >>= 1) {
            tlo = fminf(tlo, __shfl_xor_sync(0xffffffffu, tlo, d));
            thi = fmaxf(thi, __shfl_xor_sync(0xffffffffu, thi, d));
        }
        if (lane == 0) {
            red_lo[warp] = tlo;
            red_hi[warp] = thi;
        }
        __syncthreads();
        // 3. unit extremes through distributed shared memory -> bound: lane r
        // of warp 0 stores this slice's extremes into CTA r
        if (warp == 0) {
            float lo = lane < kWarps ? red_lo[lane] : FLT_MAX;
            float hi = lane < kWarps ? red_hi[lane] : -FLT_MAX;
#pragma unroll
            for (int d = 16; d > 0; d >>= 1) {
                lo = fminf(lo, __shfl_xor_sync(0xffffffffu, lo, d));
                hi = fmaxf(hi, __shfl_xor_sync(0xffffffffu, hi, d));
            }
            if (static_cast<uint32_t>(lane) < csize)
                *cluster.map_shared_rank(&s_extremes[rank], static_cast<uint32_t>(lane)) =
                    make_float2(lo, hi);
        }
        cluster.sync();
        if (warp == 0) {
            float lo = FLT_MAX, hi = -FLT_MAX;
            if (static_cast<uint32_t>(lane) < csize) {
                lo = s_extremes[lane].x;
                hi = s_extremes[lane].y;
            }
#pragma unroll
            for (int d = 16; d > 0; d >>= 1) {
                lo = fminf(lo, __shfl_xor_sync(0xffffffffu, lo, d));
                hi = fmaxf(hi, __shfl_xor_sync(0xffffffffu, hi, d));
            }
            if (lane == 0) {
                const float eb = resolve_bound(unit.eb, lo, hi, a.relative != 0);
                s_eb = eb;
                s_recip = __fdiv_rn(0.5f, eb);
            }
        }
        __syncthreads();
        const float eb = s_eb;
        const float recip = s_recip;

        // 4. rates, payload offsets (one scan for all rounds), slice size
        uint32_t off[R];
        bool any_wide = !(recip <= FLT_MAX);  // 0.5 / eb must be finite for +0 padding
#pragma unroll
        for (int k = 0; k < R; ++k) {
            const uint32_t i = k * kThreads + tid;
            uint32_t sz = 0;
            if (i < nbs) {
                float lo, hi;
                if constexpr (sizeof(T) == 2) {
                    const uint32_t p = ext16[i];
                    lo = __uint_as_float(p << 16);
                    hi = __uint_as_float(p & 0xffff0000u);
                } else {
                    lo = ext32[i].x;
                    hi = ext32[i].y;
                }
                const bool nan = rates[i] & kNanFlag;
                uint32_t m = 0;
                if (lo == lo) m = max(uabs(quantize(lo, recip)), uabs(quantize(hi, recip)));
                if (nan) m = max(m, 1u);
                const uint32_t r = 32 - __clz(m);
                rates[i] = static_cast<uint8_t>(r | (nan ? kNanFlag : 0));
                any_wide |= nan || r > 15;
                sz = r ? 4 + 4 * r : 0u;
            }
            uint32_t x = sz;
#pragma unroll
            for (int d = 1; d < 32; d <<= 1) {
                const uint32_t y = __shfl_up_sync(0xffffffffu, x, d);
                if (lane >= d) x += y;
            }
            if (lane == 31) wsum[k][warp] = x;
            off[k] = x - sz;
        }
        const bool inplace = !__syncthreads_or(any_wide);
        // every extremes word has been read: the region now holds offsets
        uint32_t slice_total = 0;
#pragma unroll
        for (int k = 0; k < R; ++k) {
            uint32_t pre = 0, tot = 0;
#pragma unroll
            for (int w = 0; w < kWarps; ++w) {
                const uint32_t s = wsum[k][w];
                pre += w < warp ? s : 0u;
                tot += s;
            }
            const uint32_t i = k * kThreads + tid;
            if (i < nbs) offs[i] = slice_total + off[k] + pre;
            slice_total += tot;
        }
        if (warp == 0 && static_cast<uint32_t>(lane) < csize)
            *cluster.map_shared_rank(&s_totals[rank], static_cast<uint32_t>(lane)) = slice_total;
        cluster.sync();
        if (warp == 0) {
            const uint32_t t = static_cast<uint32_t>(lane) < csize ? s_totals[lane] : 0u;
            uint32_t base = static_cast<uint32_t>(lane) < rank ? t : 0u, all = t;
#pragma unroll
            for (int d = 16; d > 0; d >>= 1) {
                base += __shfl_xor_sync(0xffffffffu, base, d);
                all += __shfl_xor_sync(0xffffffffu, all, d);
            }
            if (lane == 0) {
                s_base = base;
                s_unit_total = all;
            }
        }
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
            for (uint32_t i = tid; i < nbs; i += kThreads) stream[b0 + i] = rates[i] & 0x3f;
            if (rank == csize - 1)
                for (uint32_t j = nb + tid; j < hdr; j += kThreads) stream[j] = 0;

            // 5. pack round by round
            const uint64_t start = static_cast<uint64_t>(hdr) + s_base;
            const uint32_t shift =
                static_cast<uint32_t>((reinterpret_cast<uintptr_t>(stream) + start) & 15u);
            uint8_t* out_smem = smem + shift;   // slice payload byte 0 (in place)
            const uint32_t sh = 8u * rho;
            const uint32_t rounds = (nbs + kThreads - 1) / kThreads;
#pragma unroll 1
            for (uint32_t k = 0; k < rounds; ++k) {
                const uint32_t i = k * kThreads + tid;
                const bool active = i < nbs;
                const uint32_t rb = active ? rates[i] : 0u;
                const uint32_t r = rb & 0x3f;
                const uint32_t valid =
                    active ? min(n - (b0 + i) * kBlock, uint32_t(kBlock)) : uint32_t(kBlock);
                const uint32_t pos = active ? offs[i] : 0u;
                uint32_t w[Traits<T>::kWords];
                if (active) load_block<T>(slice + i * BB, rho, w);
                if (inplace) {
                    uint32_t A[16];
                    if (active) {
                        const uint32_t orv = narrow_block<T>(w, recip, A);
                        if (32u - __clz(orv >> 1) != r) status |= kErrRateCheck;
                    }
                    __syncthreads();  // every input of this round is in registers
                    if (active && r) {
                        uint32_t* out = reinterpret_cast<uint32_t*>(out_smem + pos);
#pragma unroll
                        for (int t = 0; t < 16; ++t)
                            if (t <= static_cast<int>(r)) out[t] = __funnelshift_l(A[t], A[t], sh);
                    }
                } else {
                    const bool narrow_ok = !(rb & kNanFlag) && r <= 15;
                    const bool wide = __any_sync(0xffffffffu, active && !narrow_ok);
                    if (active) {
                        uint32_t* out = reinterpret_cast<uint32_t*>(stream + start + pos);
                        uint32_t orv;
                        if (!wide) {
                            uint32_t A[16];
                            orv = narrow_block<T>(w, recip, A) >> 1;
#pragma unroll
                            for (int t = 0; t < 16; ++t)
                                if (r && t <= static_cast<int>(r))
                                    out[t] = __funnelshift_l(A[t], A[t], sh);
                        } else {
                            orv = wide_block<T>(w, rho, recip, valid, r, out);
                        }
                        if (32u - __clz(orv) != r) status |= kErrRateCheck;
                    }
                }
            }
            if (inplace) {
                fence_proxy_async_smem();
                __syncthreads();
                const uint64_t g_end = start + slice_total;
                const uint64_t a0 = (reinterpret_cast<uintptr_t>(stream) + start + 15u) & ~uint64_t(15);
                const uint64_t a1 = (reinterpret_cast<uintptr_t>(stream) + g_end) & ~uint64_t(15);
                const uint64_t s0 = reinterpret_cast<uintptr_t>(stream) + start;
                const uint64_t s1 = reinterpret_cast<uintptr_t>(stream) + g_end;
                const bool body = a1 > a0;
                const uint64_t head_end = body ? a0 : s1;
                if (body && tid == 0) {
                    bulk_store(reinterpret_cast<void*>(a0), out_smem + (a0 - s0),
                               static_cast<uint32_t>(a1 - a0));
                    bulk_commit();
                }
                const uint32_t head_words = static_cast<uint32_t>(head_end - s0) >> 2;
                const uint32_t tail_words = body ? static_cast<uint32_t>(s1 - a1) >> 2 : 0u;
                if (static_cast<uint32_t>(tid) < head_words) {
                    reinterpret_cast<uint32_t*>(s0)[tid] =
                        reinterpret_cast<const uint32_t*>(out_smem)[tid];
                } else if (tid >= 32 && static_cast<uint32_t>(tid - 32) < tail_words) {
                    const uint32_t t = tid - 32;
                    reinterpret_cast<uint32_t*>(a1)[t] =
                        reinterpret_cast<const uint32_t*>(out_smem + (a1 - s0))[t];
                }
                if (tid == 0) bulk_wait<0>();
            }
        }
        if (status) atomicOr(&s_status, status);
        __syncthreads();
        // Status lives in mapped host memory: a plain store (no atomics over
        // PCIe); any CTA that saw an error leaves a nonzero word.
        if (tid == 0 && s_status) *reinterpret_cast<volatile uint32_t*>(&a.status[u]) = s_status;
        // No CTA reads another's shared memory after the second cluster
        // barrier, and the next unit's stores into s_extremes / s_totals come
        // after barriers this CTA only reaches once it has read them.
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
    cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           L::kTotal);
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
