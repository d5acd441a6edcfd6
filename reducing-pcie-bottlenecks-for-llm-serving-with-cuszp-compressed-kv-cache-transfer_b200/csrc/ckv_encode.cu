// Persistent clustered encoder for the fixed-mode codec (sm_100a).
//
// A thread-block cluster of c CTAs (one CTA per SM) walks a list of units
// (KV pages, or the selected layers of one); every CTA of the cluster owns
// the same contiguous slice of each unit's 32-element blocks.  A slice is
// read from HBM once (TMA bulk copies into shared memory) and its compressed
// bytes are written once.  Each CTA keeps three slices in flight and splits
// its warps by role so that copies, cluster exchanges and arithmetic of
// neighbouring units overlap:
//
//   producer warp    bulk-loads slice j into buffer j % 3 as soon as unit
//                    j-3 has been packed out of it;
//   analysis warps   per unit: block min / max / NaN-presence (packed BF16
//                    min/max); slice extremes pushed into every CTA of the
//                    cluster (asynchronous distributed-shared-memory stores
//                    counted in bytes on the receiver's mbarrier) -> absolute
//                    bound eb = eps * fmaxf(max - min, 1e-6f)
//                    (cuszp_batched_fixed.cu:55-133); per block rate = bit
//                    length of max(|q(block min)|, |q(block max)|) (the
//                    quantiser is monotone; NaN contributes |q| = 1); a scan
//                    gives every block's payload offset; slice byte totals
//                    pushed into every CTA -> this slice's output offset;
//                    then the unit is handed to the pack warps;
//   pack warps       32-block chunks, dealt round-robin across units so no
//                    warp waits for another: header rate bytes; quantise,
//                    transpose into sign word + bit planes in registers,
//                    compact the chunk's payload in place over its own input
//                    (a block of rate <= 15 packs into at most the 64 bytes it
//                    came from; a warp barrier suffices), placed at the
//                    destination's offset modulo 16, and copy it out with one
//                    bulk copy (shared -> global) plus the ragged edge words.
//
// Rate <= 15 blocks without NaN (every block at REL bounds >= 1e-5 on
// two-sided data) use a quantiser that truncates with a round-toward-zero
// add of 2^23 instead of a float->int conversion; it gives the reference's
// integer for |q| < 2^15.  A chunk with any other block uses the reference's
// exact instruction sequence and is written straight to global memory.
//
// The rate found while packing from the values themselves is checked
// against the one from the extremes; a mismatch sets kErrRateCheck.  Every
// wait is bounded; a wait that runs out sets kErrTimeout on the cluster's
// units and every role stops after the copies it issued have landed.
#include "ckv_launch.h"

#include <cooperative_groups.h>

#include <atomic>
#include <cfloat>
#include <map>
#include <mutex>

namespace cg = cooperative_groups;

namespace ckv {
namespace {

constexpr uint32_t kMaxCluster = 16;
constexpr uint32_t kWaitPolls = 1u << 24;
constexpr uint32_t kMaxPieces = 512;
constexpr uint8_t kNanFlag = 0x80;
constexpr uint32_t kXSlots = 2;     // cluster exchange slots (units j and j+1)
constexpr int kPWarps = 11;         // pack warps
constexpr int kAWarps = 4;          // analysis warps
constexpr int kAThreads = kAWarps * 32;
constexpr int kProducerWarp = kPWarps + kAWarps;
constexpr int kEncThreads = (kProducerWarp + 1) * 32;
constexpr uint32_t kWaitSpins = 1u << 26;   // polls of a non-suspending wait
// Whole BF16 pages of at most this many elements take the streaming encoder
// by default: measured on B200, it is faster there (8192: 1.3-1.45x, 16384:
// 1.05-1.15x) and slower from 32768 elements up (C2 pages: 0.86x).
constexpr uint32_t kStreamMaxElems = 16384;

// Slice geometry of a launch: bytes of one CTA's slice of a unit, slices
// (and per-unit metadata sets) in flight per CTA, and the blocks per
// analysis thread in the offset scan.  Units of up to nine 64 KB slices use
// three 64 KB buffers; larger units two 100 KB buffers, so that their
// clusters stay at nine CTAs or fewer (B200 keeps 15 clusters of 7-9 CTAs
// resident but only 7 of 11-16: 135 SMs against 112).
struct Geo64 {
    static constexpr uint32_t kSliceBytes = 64 * 1024;
    static constexpr uint32_t kBufs = 3;
    static constexpr uint32_t kMaxRun = 8;
    static constexpr uint32_t kMetaStride = 4096;
};
struct Geo100 {
    static constexpr uint32_t kSliceBytes = 100 * 1024;
    static constexpr uint32_t kBufs = 2;
    static constexpr uint32_t kMaxRun = 13;
    static constexpr uint32_t kMetaStride = 6400;
};

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

// Dynamic shared memory: kBufs slices, then kBufs x block extremes (later
// payload offsets, 4 bytes a block either type), then kBufs x rate bytes.
template <typename T, typename G>
struct Layout {
    static constexpr uint32_t kBufs = G::kBufs;
    static constexpr uint32_t kSliceBytes = G::kSliceBytes;
    static constexpr uint32_t kMaxRun = G::kMaxRun;
    static constexpr uint32_t kBlocks = kSliceBytes / (kBlock * Traits<T>::kBytes);
    static constexpr uint32_t kMeta = kBufs * kSliceBytes;
    static constexpr uint32_t kMetaStride = G::kMetaStride;
    static constexpr uint32_t kRates = kMeta + kBufs * kMetaStride;
    static constexpr uint32_t kRatesStride = (kBlocks + 15) / 16 * 16;
    static constexpr uint32_t kTotal = kRates + kBufs * kRatesStride;
    static_assert(kBlocks * 4 <= kMetaStride, "offsets per slice");
    static_assert(kBlocks <= kAThreads * kMaxRun, "offset scan");
};

struct EncodeArgs {
    const Unit* units;
    const Map* maps;
    uint32_t num_units;
    uint32_t relative;
    uint64_t* sizes;
    float* bounds;
    uint32_t* status;
    ShiftMul mul;
    // Failure-path test hook: the cluster that owns unit withhold_unit
    // (~0u: none) never completes that unit's bound exchange, and its waits
    // on other roles and CTAs give up after test_polls polls.
    uint32_t withhold_unit;
    uint32_t test_polls;
};

// Poll limits of one CTA's waits on other roles and CTAs.
struct Limits {
    uint32_t polls;   // suspending waits (mbarrier try_wait)
    uint32_t spins;   // non-suspending waits (cluster exchanges)
};

// This CTA's share of a unit of n elements.
struct Slice {
    uint32_t n, nb, b0, nbs, e0, e1, hdr;
};

__device__ __forceinline__ Slice slice_of(uint32_t n, uint32_t rank, uint32_t csize) {
    Slice s;
    s.n = n;
    s.nb = (n + kBlock - 1) / kBlock;
    const uint32_t sb = (s.nb + csize - 1) / csize;
    s.b0 = min(rank * sb, s.nb);
    const uint32_t b1 = min(s.b0 + sb, s.nb);
    s.nbs = b1 - s.b0;
    s.e0 = s.b0 * kBlock;
    s.e1 = min(b1 * kBlock, n);
    s.hdr = (n + kGroup - 1) / kGroup * (kGroup / kBlock);
    return s;
}

// What the analysis warps hand to the pack warps (and, through them, to
// the producer) for one unit.
struct SetInfo {
    uint8_t* stream;      // the unit's compressed stream
    uint8_t* out;         // this slice's payload in it
    uint64_t unit_bytes;  // compressed size of the unit
    float eb, recip;      // bound, 0.5 / eb
    uint32_t n, b0, nbs;
    uint32_t pad_from, pad_to;   // header bytes after the last block (last CTA)
    uint32_t fits;
};

// One unit as the producer publishes it with the slice load.
struct Job {
    uint8_t* stream;
    uint64_t capacity;
    float eps;
    uint32_t u;
    Slice s;
};

// Barriers and exchange slots of one CTA.
template <typename G>
struct Sync {
    static constexpr uint32_t kBufs = G::kBufs;
    uint64_t full[kBufs];      // producer -> analysis: slice landed
    uint64_t ready[kBufs];     // analysis -> pack: offsets, bound, output address
    uint64_t packed[kBufs];    // pack warps -> producer: buffer and metadata free
    uint64_t ext_bar[kXSlots]; // cluster: slice extremes of every CTA stored here
    uint64_t tot_bar[kXSlots]; // cluster: slice byte totals of every CTA stored here
    SetInfo info[kBufs];
    Job job[kBufs];
    uint32_t tail[kBufs];
    uint32_t status[kBufs];
    // Written by every CTA of the cluster into every CTA (asynchronous
    // distributed shared memory stores counted on the receiver's barrier).
    float2 ext[kXSlots][kMaxCluster];
    uint32_t tot[kXSlots][kMaxCluster];
    float red_lo[kAWarps], red_hi[kAWarps];
    uint32_t scan[kAWarps];
    uint32_t broken;
};

// Barrier of the analysis warps.
__device__ __forceinline__ void abar() {
    asm volatile("bar.sync 1, %0;" ::"n"(kAThreads) : "memory");
}

// Barrier of the analysis warps that also ORs a predicate over them, so
// that every analysis thread takes the same branch on a flag that other
// roles may set at any time.
__device__ __forceinline__ bool abar_or(bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.or.pred q, 1, %2, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"(static_cast<uint32_t>(v)), "n"(kAThreads)
        : "memory");
    return r != 0;
}

// ---- slice load (producer lane) ----------------------------------------------

// Plans the load of elements [e0, e1) as bulk copies of 16-byte aligned runs
// and issues them on `bar`.  *tail (written before the arrive, so it is
// visible once the phase completes) is the first element the compute warps
// copy themselves: the sub-16-byte tail, or e0 when some run cannot be
// bulk-copied.
template <typename T>
__device__ void issue_load(const Unit& unit, const Map& m, uint32_t u, uint32_t e0, uint32_t e1,
                           uint8_t* slice, uint64_t* bar, volatile uint32_t* tail) {
    constexpr uint32_t B = Traits<T>::kBytes;
    const uint32_t L = run_len(unit, m);
    uint32_t total = 0, pieces = 0, t = e1;
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
        if (last) t = pos + body / B;
        pos += len;
    }
    if (!ok) {
        *tail = e0;
        mbar_arrive_expect_tx(bar, 0);
        return;
    }
    *tail = t;
    mbar_arrive_expect_tx(bar, total);
    for (uint32_t pos = e0; pos < e1;) {
        const uint32_t r = pos / L, off = pos - r * L;
        const uint32_t len = min(e1 - pos, L - off);
        const T* src = run_base<const T>(unit, m, u, r) + off;
        const uint32_t body = (len * B) & ~15u;
        if (body) bulk_load(slice + (pos - e0) * B, src, body, bar);
        pos += len;
    }
}

template <typename T>
__device__ void copy_elements(const Unit& unit, const Map& m, uint32_t u, uint32_t from,
                              uint32_t to, uint32_t e0, uint8_t* slice, uint32_t t) {
    const uint32_t L = run_len(unit, m);
    T* dst = reinterpret_cast<T*>(slice);
    for (uint32_t i = from + t; i < to; i += kAThreads) {
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

// Two rows (|q| << 1) | sign, for |q| < 2^15 and no NaN, packed as the low
// and high halves of one word, as batch_quantization
// (cuszp_batched_fixed.cu:10-25) computes q: r = x * recip and t = r + 0.5,
// each rounded; trunc(|t|) from a round-toward-zero add of 2^23 (exact for
// |t| < 2^23; the float's low 16 bits are then trunc(|t|)).  The reference's
// s = (r < -0.5) is the sign bit of t: r + 0.5 is exact for r in [-1, -0.5)
// (Sterbenz), so t < 0 exactly when r < -0.5, and t is never -0.  Then
// |q| = trunc(|t|) + s and the row is 2 * trunc(|t|) + 3 * s (< 2^16, so the
// halves never carry into each other): one byte permute gathers both
// truncations, one sign-replicating byte permute both signs, and one
// multiply-add forms both rows.  The two rows' multiplies are one packed
// mul.rn.f32x2 and their adds one packed fma.rn.f32x2(r, 1, 0.5), which is
// r + 0.5 rounded once: ptxas keeps a packed multiply and that FMA apart,
// whereas it contracts a packed multiply followed by add.rn.f32x2 into one
// fused multiply-add despite the rounding modifiers (the fma_probe golden
// case catches that).  Each lane rounds as its scalar form does.
// prmt.b32 in its default mode, where a selector nibble of 8-15 replicates
// the sign bit of byte (nibble & 7) over the result byte (the __byte_perm
// intrinsic uses only the low 3 bits of each nibble).
__device__ __forceinline__ uint32_t prmt_sign(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

__device__ __forceinline__ uint32_t narrow_pair(float x_lo, float x_hi, uint64_t recip2,
                                                const ShiftMul& mul) {
    uint64_t x2, r2, t2;
    asm("mov.b64 %0, {%1, %2};" : "=l"(x2) : "f"(x_lo), "f"(x_hi));
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r2) : "l"(x2), "l"(recip2));
    asm("fma.rn.f32x2 %0, %1, %2, %3;"
        : "=l"(t2)
        : "l"(r2), "l"(0x3F8000003F800000ull), "l"(0x3F0000003F000000ull));
    float t_lo, t_hi;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(t_lo), "=f"(t_hi) : "l"(t2));
    const float z_lo = __fadd_rz(fabsf(t_lo), 8388608.0f);
    const float z_hi = __fadd_rz(fabsf(t_hi), 8388608.0f);
    const uint32_t trunc2 = __byte_perm(__float_as_uint(z_lo), __float_as_uint(z_hi), 0x5410);
    // 0xffff in each half whose t is negative
    const uint32_t neg2 = prmt_sign(__float_as_uint(t_lo), __float_as_uint(t_hi), 0xffbbu);
    return trunc2 * mul.l1 + (neg2 & 0x00030003u);
}

// Rows of the 16x32 bit matrix for a narrow block: A[k] holds rows k and
// k + 16, then the transpose turns them into the sign word (A[0]) and the
// planes (A[1 + b]).  Elements past the end of the unit were set to +0 in
// shared memory, which quantises to 0 for a finite 0.5 / eb.  Returns the
// OR of all rows.
template <typename T>
__device__ __forceinline__ uint32_t narrow_block(const uint32_t (&w)[Traits<T>::kWords],
                                                 float recip, const ShiftMul& mul,
                                                 uint32_t (&A)[16]) {
    uint32_t orv = 0;
    uint64_t recip2;
    asm("mov.b64 %0, {%1, %1};" : "=l"(recip2) : "f"(recip));
#pragma unroll
    for (int k = 0; k < 16; ++k) {
        const int e = bitpos(k);
        A[k] = narrow_pair(elem<T>(w, e), elem<T>(w, e + 16), recip2, mul);
        orv |= A[k];
    }
    transpose16_mul<true, true>(A, mul);
    return (orv | (orv >> 16)) & 0xffffu;
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

// Minimum and maximum of a block's values that are not NaN, and whether any
// is NaN.  BF16: the maximum tree propagates NaN, so one tree gives both the
// maximum and the NaN flag; a block with a NaN (rare) takes a second,
// NaN-ignoring maximum tree.
template <typename T>
__device__ __forceinline__ void block_extremes(const uint32_t (&w)[Traits<T>::kWords], float& lo,
                                               float& hi, bool& nan);

template <>
__device__ __forceinline__ void block_extremes<__nv_bfloat16>(const uint32_t (&w)[16], float& lo,
                                                              float& hi, bool& nan) {
    __nv_bfloat162 mn[8], mz[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(&w[2 * k]);
        const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&w[2 * k + 1]);
        mn[k] = __hmin2(a, b);
        mz[k] = __hmax2_nan(a, b);
    }
#pragma unroll
    for (int s = 4; s >= 1; s >>= 1) {
#pragma unroll
        for (int k = 0; k < s; ++k) {
            mn[k] = __hmin2(mn[k], mn[k + s]);
            mz[k] = __hmax2_nan(mz[k], mz[k + s]);
        }
    }
    lo = fminf(__low2float(mn[0]), __high2float(mn[0]));
    const float a = __low2float(mz[0]), b = __high2float(mz[0]);
    nan = (a != a) || (b != b);
    hi = fmaxf(a, b);
    if (nan) {   // the maximum over the values that are not NaN
        __nv_bfloat162 mx[8];
#pragma unroll
        for (int k = 0; k < 8; ++k)
            mx[k] = __hmax2(*reinterpret_cast<const __nv_bfloat162*>(&w[2 * k]),
                            *reinterpret_cast<const __nv_bfloat162*>(&w[2 * k + 1]));
#pragma unroll
        for (int s = 4; s >= 1; s >>= 1) {
#pragma unroll
            for (int k = 0; k < s; ++k) mx[k] = __hmax2(mx[k], mx[k + s]);
        }
        hi = fmaxf(__low2float(mx[0]), __high2float(mx[0]));
    }
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

// ---- producer warp (one lane) -------------------------------------------------

// Loads slice j into buffer j % kBufs once unit j - kBufs has been packed out
// of it, and publishes each unit's status word after its pack.  Returns once
// the copies it issued have landed.
template <typename T, typename G>
__device__ void produce(const EncodeArgs& a, const Limits& lim, uint32_t count, uint32_t first,
                        uint32_t stride, uint32_t rank, uint32_t csize, uint8_t* smem, Sync<G>& sy) {
    uint32_t last[G::kBufs];
    for (uint32_t b = 0; b < G::kBufs; ++b) last[b] = ~0u;
    for (uint32_t j = 0; j < count + G::kBufs; ++j) {
        const uint32_t b = j % G::kBufs;
        if (j >= G::kBufs) {
            const uint32_t jj = j - G::kBufs;
            if (!mbar_wait_bounded(&sy.packed[b], (jj / G::kBufs) & 1u, lim.polls)) {
                sy.broken = 1;
                break;
            }
            // Results live in mapped host memory.  They are written here, by a
            // lane that never releases at cluster scope, so that no
            // exchange waits for a PCIe write.  Status is a plain store (no
            // atomics over PCIe); any CTA that saw an error leaves a nonzero
            // word.
            const uint32_t uj = first + jj * stride;
            if (rank == 0) {
                a.sizes[uj] = sy.info[b].unit_bytes;
                a.bounds[uj] = sy.info[b].eb;
            }
            if (sy.status[b]) *reinterpret_cast<volatile uint32_t*>(&a.status[uj]) = sy.status[b];
            sy.status[b] = 0;
        }
        if (j < count) {
            const uint32_t u = first + j * stride;
            const Unit unit = a.units[u];
            const Map map = a.maps[unit.map];
            const Slice s = slice_of(unit.n, rank, csize);
            Job& job = sy.job[b];
            job.stream = unit.stream;
            job.capacity = unit.capacity;
            job.eps = unit.eb;
            job.u = u;
            job.s = s;
            // published by the arrive on full[b] inside issue_load
            issue_load<T>(unit, map, u, s.e0, s.e1, smem + b * G::kSliceBytes, &sy.full[b],
                          &sy.tail[b]);
            last[b] = j;
        }
    }
    for (uint32_t b = 0; b < G::kBufs; ++b)
        if (last[b] != ~0u) mbar_wait_bounded(&sy.full[b], (last[b] / G::kBufs) & 1u, kWaitPolls);
}

// ---- analysis warps -------------------------------------------------------------

template <typename T, typename G>
__device__ void analyse(const EncodeArgs& a, const Limits& lim, uint32_t count, uint32_t first,
                        uint32_t stride, cg::cluster_group& cluster, uint8_t* smem, Sync<G>& sy) {
    using L = Layout<T, G>;
    constexpr uint32_t BB = kBlock * Traits<T>::kBytes;  // input bytes per block
    const uint32_t rank = cluster.block_rank();
    const uint32_t csize = cluster.num_blocks();
    const uint32_t t = threadIdx.x - kPWarps * 32;
    const int lane = t & 31, awarp = t >> 5;
    const int rho = (sizeof(T) == 2) ? ((t >> 1) & 3) : (t & 3);
    for (uint32_t j = 0; j < count; ++j) {
        const uint32_t b = j % G::kBufs, x = j % kXSlots;
        const uint32_t xpar = (j / kXSlots) & 1u;
        uint8_t* slice = smem + b * G::kSliceBytes;
        uint8_t* meta = smem + L::kMeta + b * L::kMetaStride;
        uint8_t* rates = smem + L::kRates + b * L::kRatesStride;

        // -- slice on chip, block extremes, slice extremes to the cluster
        const bool landed = mbar_wait_bounded(&sy.full[b], (j / G::kBufs) & 1u, lim.polls);
        const Job job = sy.job[b];
        const Slice& s = job.s;
        const uint32_t u = job.u;
        if (landed) {
            const uint32_t tail = sy.tail[b];
            if (tail < s.e1) {   // runs the bulk copies could not take
                const Unit unit = a.units[u];
                copy_elements<T>(unit, a.maps[unit.map], u, tail, s.e1, s.e0, slice, t);
            }
            // +0 past the end of the unit (the last block may be partial)
            if (s.nbs && s.b0 + s.nbs == s.nb && t < s.nb * kBlock - s.e1)
                reinterpret_cast<T*>(slice)[s.e1 - s.e0 + t] = T(0.0f);
        } else {
            sy.broken = 1;
        }
        if (abar_or(*reinterpret_cast<volatile uint32_t*>(&sy.broken) != 0)) return;
        float tlo = FLT_MAX, thi = -FLT_MAX;
        // Full blocks four at a time: every load of a group is issued before
        // its stores (which the compiler cannot move across later loads).
        const uint32_t nfull = min(s.nbs, (s.n - s.e0) / kBlock);
        uint32_t i = t;
        for (; i + 3 * kAThreads < nfull; i += 4 * kAThreads) {
            uint32_t w[4][Traits<T>::kWords];
#pragma unroll
            for (int g = 0; g < 4; ++g) load_block<T>(slice + (i + g * kAThreads) * BB, rho, w[g]);
            float lo[4], hi[4];
            bool nan[4];
#pragma unroll
            for (int g = 0; g < 4; ++g) block_extremes<T>(w[g], lo[g], hi[g], nan[g]);
#pragma unroll
            for (int g = 0; g < 4; ++g) {
                const uint32_t ig = i + g * kAThreads;
                if constexpr (sizeof(T) == 2)
                    reinterpret_cast<uint32_t*>(meta)[ig] =
                        (__float_as_uint(lo[g]) >> 16) | (__float_as_uint(hi[g]) & 0xffff0000u);
                else
                    reinterpret_cast<float2*>(meta)[ig] = make_float2(lo[g], hi[g]);
                rates[ig] = nan[g] ? kNanFlag : 0;
                tlo = fminf(tlo, lo[g]);
                thi = fmaxf(thi, hi[g]);
            }
        }
        for (; i < s.nbs; i += kAThreads) {
            const uint8_t* blk = slice + i * BB;
            float lo, hi;
            bool nan;
            const uint32_t valid = min(s.n - (s.b0 + i) * kBlock, uint32_t(kBlock));
            if (valid == kBlock) {
                uint32_t w[Traits<T>::kWords];
                load_block<T>(blk, rho, w);
                block_extremes<T>(w, lo, hi, nan);
            } else {
                lo = __int_as_float(0x7fffffff);
                hi = lo;
                nan = false;
                for (uint32_t v = 0; v < valid; ++v) {
                    const float xv = elem_at<T>(blk, v);
                    lo = fminf(lo, xv);
                    hi = fmaxf(hi, xv);
                    nan |= xv != xv;
                }
            }
            if constexpr (sizeof(T) == 2)
                reinterpret_cast<uint32_t*>(meta)[i] =
                    (__float_as_uint(lo) >> 16) | (__float_as_uint(hi) & 0xffff0000u);
            else
                reinterpret_cast<float2*>(meta)[i] = make_float2(lo, hi);
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
            sy.red_lo[awarp] = tlo;
            sy.red_hi[awarp] = thi;
        }
        abar();
        if (awarp == 0) {
            float lo = lane < kAWarps ? sy.red_lo[lane] : FLT_MAX;
            float hi = lane < kAWarps ? sy.red_hi[lane] : -FLT_MAX;
#pragma unroll
            for (int d = 16; d > 0; d >>= 1) {
                lo = fminf(lo, __shfl_xor_sync(0xffffffffu, lo, d));
                hi = fmaxf(hi, __shfl_xor_sync(0xffffffffu, hi, d));
            }
            if (lane == 0) mbar_arrive_expect_tx(&sy.ext_bar[x], csize * sizeof(float2));
            if (static_cast<uint32_t>(lane) < csize && !(u == a.withhold_unit && rank == 0))
                st_async_f32x2(cluster_addr(&sy.ext[x][rank], lane), lo, hi,
                               cluster_addr(&sy.ext_bar[x], lane));
            // -- unit extremes -> bound
            const bool ok =
                __all_sync(0xffffffffu, mbar_spin_bounded(&sy.ext_bar[x], xpar, lim.spins));
            lo = FLT_MAX;
            hi = -FLT_MAX;
            if (static_cast<uint32_t>(lane) < csize) {
                lo = sy.ext[x][lane].x;
                hi = sy.ext[x][lane].y;
            }
#pragma unroll
            for (int d = 16; d > 0; d >>= 1) {
                lo = fminf(lo, __shfl_xor_sync(0xffffffffu, lo, d));
                hi = fmaxf(hi, __shfl_xor_sync(0xffffffffu, hi, d));
            }
            if (lane == 0) {
                if (!ok) sy.broken = 1;
                const float eb = resolve_bound(job.eps, lo, hi, a.relative != 0);
                sy.info[b].eb = eb;
                sy.info[b].recip = __fdiv_rn(0.5f, eb);
            }
        }
        if (abar_or(*reinterpret_cast<volatile uint32_t*>(&sy.broken) != 0)) return;

        // -- rates and payload offsets: each thread a run of kRun blocks
        const float recip = sy.info[b].recip;
        const uint32_t run = (s.nbs + kAThreads - 1) / kAThreads;
        const uint32_t i0 = t * run;
        // every load of the run first, then the arithmetic, then the stores
        float lo[G::kMaxRun], hi[G::kMaxRun];
        uint32_t flag[G::kMaxRun], sz[G::kMaxRun];
#pragma unroll
        for (uint32_t k = 0; k < G::kMaxRun; ++k) {
            lo[k] = hi[k] = 0.0f;
            flag[k] = 0;
            const uint32_t ik = i0 + k;
            if (k < run && ik < s.nbs) {
                if constexpr (sizeof(T) == 2) {
                    const uint32_t p = reinterpret_cast<const uint32_t*>(meta)[ik];
                    lo[k] = __uint_as_float(p << 16);
                    hi[k] = __uint_as_float(p & 0xffff0000u);
                } else {
                    const float2 p = reinterpret_cast<const float2*>(meta)[ik];
                    lo[k] = p.x;
                    hi[k] = p.y;
                }
                flag[k] = rates[ik] & kNanFlag;
            }
        }
        uint32_t local = 0;
#pragma unroll
        for (uint32_t k = 0; k < G::kMaxRun; ++k) {
            uint32_t mq = 0;
            if (lo[k] == lo[k]) mq = max(uabs(quantize(lo[k], recip)), uabs(quantize(hi[k], recip)));
            if (flag[k]) mq = max(mq, 1u);
            const uint32_t r = 32 - __clz(mq);
            const bool in = k < run && i0 + k < s.nbs;
            sz[k] = in && r ? 4 + 4 * r : 0u;
            flag[k] |= r;
            local += sz[k];
        }
#pragma unroll
        for (uint32_t k = 0; k < G::kMaxRun; ++k)
            if (k < run && i0 + k < s.nbs) rates[i0 + k] = static_cast<uint8_t>(flag[k]);
        uint32_t inc = local;
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            const uint32_t y = __shfl_up_sync(0xffffffffu, inc, d);
            if (lane >= d) inc += y;
        }
        if (lane == 31) sy.scan[awarp] = inc;
        abar();
        uint32_t pre = 0, slice_total = 0;
#pragma unroll
        for (int w = 0; w < kAWarps; ++w) {
            const uint32_t v = sy.scan[w];
            pre += w < awarp ? v : 0u;
            slice_total += v;
        }
        // The extremes of these blocks were read by this thread only: the
        // words now hold payload offsets.
        uint32_t off = pre + inc - local;
#pragma unroll
        for (uint32_t k = 0; k < G::kMaxRun; ++k) {
            if (k < run && i0 + k < s.nbs) reinterpret_cast<uint32_t*>(meta)[i0 + k] = off;
            off += sz[k];
        }
        if (awarp == 0) {
            if (lane == 0) mbar_arrive_expect_tx(&sy.tot_bar[x], csize * sizeof(uint32_t));
            if (static_cast<uint32_t>(lane) < csize)
                st_async_u32(cluster_addr(&sy.tot[x][rank], lane), slice_total,
                             cluster_addr(&sy.tot_bar[x], lane));
            // -- slice totals -> this slice's output offset
            const bool ok =
                __all_sync(0xffffffffu, mbar_spin_bounded(&sy.tot_bar[x], xpar, lim.spins));
            const uint32_t tv = static_cast<uint32_t>(lane) < csize ? sy.tot[x][lane] : 0u;
            uint32_t base = static_cast<uint32_t>(lane) < rank ? tv : 0u, all = tv;
#pragma unroll
            for (int d = 16; d > 0; d >>= 1) {
                base += __shfl_xor_sync(0xffffffffu, base, d);
                all += __shfl_xor_sync(0xffffffffu, all, d);
            }
            if (lane == 0) {
                if (!ok) sy.broken = 1;
                const uint64_t unit_bytes = static_cast<uint64_t>(s.hdr) + all;
                const bool fits = unit_bytes <= job.capacity;
                if (!fits) sy.status[b] |= kErrCapacity;
                SetInfo& info = sy.info[b];
                info.stream = job.stream;
                info.out = job.stream + s.hdr + base;
                info.unit_bytes = unit_bytes;
                info.n = s.n;
                info.b0 = s.b0;
                info.nbs = s.nbs;
                info.pad_from = rank == csize - 1 ? s.nb : 0u;
                info.pad_to = rank == csize - 1 ? s.hdr : 0u;
                info.fits = fits ? 1u : 0u;
            }
        }
        if (abar_or(*reinterpret_cast<volatile uint32_t*>(&sy.broken) != 0)) return;
        if (t == 0) mbar_arrive(&sy.ready[b]);   // offsets, bound and address published
    }
}

// ---- pack warps ----------------------------------------------------------------

// A warp copies `words` words from shared to global memory, four loads in
// flight per lane before their stores.
__device__ __forceinline__ void copy_out(const uint32_t* src, uint32_t* dst, uint32_t words,
                                         int lane) {
    for (uint32_t k = lane; k < words; k += 128) {
        uint32_t v[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) v[t] = k + 32 * t < words ? src[k + 32 * t] : 0u;
#pragma unroll
        for (int t = 0; t < 4; ++t)
            if (k + 32 * t < words) dst[k + 32 * t] = v[t];
    }
}

template <typename T, typename G>
__device__ void pack(const Limits& lim, uint32_t count, const ShiftMul& mul, uint8_t* smem,
                     Sync<G>& sy) {
    using L = Layout<T, G>;
    constexpr uint32_t BB = kBlock * Traits<T>::kBytes;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int rho = (sizeof(T) == 2) ? ((lane >> 1) & 3) : (lane & 3);
    const uint32_t sh = 8u * rho;
    uint32_t rot = 0;   // chunk c of this unit goes to pack warp (c + rot) % kPWarps
    for (uint32_t j = 0; j < count; ++j) {
        const uint32_t b = j % G::kBufs;
        const bool ok = mbar_wait_bounded(&sy.ready[b], (j / G::kBufs) & 1u, lim.polls);
        if (!__all_sync(0xffffffffu, ok)) {
            sy.broken = 1;
            if (lane == 0) bulk_wait<0>();
            return;
        }
        const SetInfo info = sy.info[b];
        uint8_t* slice = smem + b * G::kSliceBytes;
        const uint32_t* offs = reinterpret_cast<const uint32_t*>(smem + L::kMeta + b * L::kMetaStride);
        const uint8_t* rates = smem + L::kRates + b * L::kRatesStride;
        const uint32_t chunks = (info.nbs + 31) / 32;
        uint32_t status = 0;
        if (info.fits) {
            const float recip = info.recip;
            // header bytes past the last block (zero) by the warp of chunk 0
            if (static_cast<uint32_t>(warp) == rot)
                for (uint32_t k = info.pad_from + lane; k < info.pad_to; k += 32) info.stream[k] = 0;
            for (uint32_t c = (warp + kPWarps - rot) % kPWarps; c < chunks; c += kPWarps) {
                const uint32_t i = c * 32 + lane;
                const bool active = i < info.nbs;
                const uint32_t rb = active ? rates[i] : 0u;
                const uint32_t r = rb & 0x3f;
                if (active) info.stream[info.b0 + i] = static_cast<uint8_t>(r);
                const uint32_t pos = active ? offs[i] : 0u;
                uint8_t* chunk = slice + c * 32 * BB;
                uint32_t w[Traits<T>::kWords];
                if (active) load_block<T>(chunk + lane * BB, rho, w);
                const bool narrow_ok = !(rb & kNanFlag) && r <= 15;
                // +0 padding quantises to 0 only for a finite 0.5 / eb; an
                // infinite bound (0.5 / eb == 0) turns an infinite value into
                // NaN * 0, |q| = 1, which the rate from the extremes does not
                // flag as NaN
                const bool wide = __any_sync(0xffffffffu, active && !narrow_ok) ||
                                  !(recip <= FLT_MAX) || recip == 0.0f;
                if (!wide) {
                    uint32_t A[16];
                    if (active) {
                        const uint32_t orv = narrow_block<T>(w, recip, mul, A);
                        if (32u - __clz(orv >> 1) != r) status |= kErrRateCheck;
                    }
                    // Every input of the chunk is in registers: its payload is
                    // compacted over the chunk's own input, then copied out --
                    // by one bulk copy where the payload, placed at the same
                    // offset modulo 16 as its global destination, still fits
                    // the chunk's bytes (the ragged first and last words by
                    // lanes).
                    __syncwarp();
                    const uint32_t p0 = __shfl_sync(0xffffffffu, pos, 0);
                    const uint32_t end =
                        __reduce_max_sync(0xffffffffu, active && r ? pos + 4 + 4 * r : 0u);
                    const uint32_t bytes = end > p0 ? end - p0 : 0u;
                    uint8_t* gdst = info.out + p0;
                    const uint32_t shift =
                        static_cast<uint32_t>(reinterpret_cast<uintptr_t>(gdst) & 15u);
                    const bool bulk = bytes >= 64 && shift + bytes <= 32 * BB;
                    uint8_t* sbase = chunk + (bulk ? shift : 0u);
                    if (active && r) {
                        uint32_t* out = reinterpret_cast<uint32_t*>(sbase + (pos - p0));
#pragma unroll
                        for (int k = 0; k < 16; ++k)
                            if (k <= static_cast<int>(r)) out[k] = __funnelshift_l(A[k], A[k], sh);
                    }
                    if (bulk) {
                        const uint32_t head = (16u - shift) & 15u;
                        const uint32_t body = (bytes - head) & ~15u;
                        const uint32_t tail = bytes - head - body;
                        fence_proxy_async_smem();   // the lanes' stores, to the bulk copy
                        __syncwarp();
                        const uint32_t* s32 = reinterpret_cast<const uint32_t*>(sbase);
                        uint32_t* g32 = reinterpret_cast<uint32_t*>(gdst);
                        if (static_cast<uint32_t>(lane) < head / 4) g32[lane] = s32[lane];
                        if (lane >= 4 && static_cast<uint32_t>(lane - 4) < tail / 4) {
                            const uint32_t w = (head + body) / 4 + (lane - 4);
                            g32[w] = s32[w];
                        }
                        if (lane == 0) {
                            bulk_store(gdst + head, sbase + head, body);
                            bulk_commit();
                        }
                    } else {
                        __syncwarp();
                        copy_out(reinterpret_cast<const uint32_t*>(chunk),
                                 reinterpret_cast<uint32_t*>(info.out + p0), bytes >> 2, lane);
                    }
                } else if (active) {
                    const uint32_t valid = min(info.n - (info.b0 + i) * kBlock, uint32_t(kBlock));
                    uint32_t* out = reinterpret_cast<uint32_t*>(info.out + pos);
                    const uint32_t orv = wide_block<T>(w, rho, recip, valid, r, out);
                    if (32u - __clz(orv) != r) status |= kErrRateCheck;
                }
            }
        }
        rot = (rot + chunks) % kPWarps;
        status = __reduce_or_sync(0xffffffffu, status);
        // Every lane's reads of this buffer, and the reads of the bulk
        // copies lane 0 issued, are done before lane 0 releases it.
        __syncwarp();
        if (lane == 0) {
            bulk_wait_read<0>();
            if (status) atomicOr(&sy.status[b], status);
            mbar_arrive(&sy.packed[b]);
        }
    }
    if (lane == 0) bulk_wait<0>();
}

// ---- the kernel --------------------------------------------------------------

template <typename T, typename G>
__global__ void __launch_bounds__(kEncThreads, 1) encode_kernel(EncodeArgs a) {
    constexpr uint32_t kBufs = G::kBufs;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ Sync<G> sy;

    cg::cluster_group cluster = cg::this_cluster();
    const uint32_t rank = cluster.block_rank();
    const uint32_t csize = cluster.num_blocks();
    const int tid = threadIdx.x, warp = tid >> 5;
    const uint32_t first = blockIdx.y, stride = gridDim.y;
    const uint32_t count =
        first < a.num_units ? (a.num_units - first + stride - 1) / stride : 0u;
    const bool tested = a.withhold_unit != ~0u && first == a.withhold_unit % stride;
    const Limits lim{tested ? a.test_polls : kWaitPolls, tested ? a.test_polls : kWaitSpins};

    if (tid == 0) {
        for (uint32_t b = 0; b < kBufs; ++b) {
            mbar_init(&sy.full[b], 1);
            mbar_init(&sy.ready[b], 1);
            mbar_init(&sy.packed[b], kPWarps);
            sy.status[b] = 0;
        }
        for (uint32_t x = 0; x < kXSlots; ++x) {
            mbar_init(&sy.ext_bar[x], 1);   // armed locally, completed by peers' bytes
            mbar_init(&sy.tot_bar[x], 1);
        }
        sy.broken = 0;
        fence_mbar_init();
    }
    cluster_barrier();   // every barrier of the cluster initialised before any arrive
    // A streaming-encoder launch of the batch's remainder units, queued after
    // this one as a programmatic dependent, may start on the SMs no cluster
    // holds once every CTA here is resident (it reads nothing written here).
    if (threadIdx.x == 0) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    if (warp == kProducerWarp) {
        if ((tid & 31) == 0) produce<T, G>(a, lim, count, first, stride, rank, csize, smem, sy);
    } else if (warp >= kPWarps) {
        analyse<T, G>(a, lim, count, first, stride, cluster, smem, sy);
    } else {
        pack<T, G>(lim, count, a.mul, smem, sy);
    }
    // No peer touches this CTA's shared memory once every CTA is here.
    cluster_barrier();
    if (tid == 0 && sy.broken)
        for (uint32_t j = 0; j < count; ++j)
            *reinterpret_cast<volatile uint32_t*>(&a.status[first + j * stride]) = kErrTimeout;
}

// Cluster size for units of at least c_min slices: the size in
// [c_min, kMaxCluster] whose co-resident clusters cover the most SMs (one
// CTA per SM), and how many clusters that is.  Cached per device.
struct ClusterShape {
    uint32_t c;
    uint32_t clusters;
};

template <typename T, typename G>
cudaError_t cluster_shape(uint32_t c_min, ClusterShape* out) {
    static std::mutex mu;
    static std::map<uint64_t, ClusterShape> cache;
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) return err;
    const uint64_t key = (static_cast<uint64_t>(dev) << 8) | c_min;
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) {
        *out = it->second;
        return cudaSuccess;
    }
    using L = Layout<T, G>;
    auto kernel = encode_kernel<T, G>;
    err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kTotal);
    if (err != cudaSuccess) return err;
    err = cudaFuncSetAttribute(kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (err != cudaSuccess) return err;
    ClusterShape best{0, 0};
    for (uint32_t c = c_min; c <= kMaxCluster; ++c) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(c, 1, 1);
        cfg.blockDim = dim3(kEncThreads, 1, 1);
        cfg.dynamicSmemBytes = L::kTotal;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = c;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int clusters = 0;
        if (cudaOccupancyMaxActiveClusters(&clusters, kernel, &cfg) != cudaSuccess) {
            cudaGetLastError();
            continue;
        }
        if (clusters > 0 && static_cast<uint64_t>(clusters) * c > static_cast<uint64_t>(best.clusters) * best.c)
            best = ClusterShape{c, static_cast<uint32_t>(clusters)};
    }
    if (best.c == 0) return cudaErrorInvalidConfiguration;
    cache[key] = best;
    *out = best;
    return cudaSuccess;
}

// Slices of a unit of nb blocks under geometry G (0 when it does not fit a
// cluster).
template <typename T, typename G>
uint32_t slices_for(uint32_t nb) {
    const uint32_t c = (nb + Layout<T, G>::kBlocks - 1) / Layout<T, G>::kBlocks;
    return c == 0 ? 1u : (c <= kMaxCluster ? c : 0u);
}

template <typename T, typename G>
cudaError_t launch_encode_g(const EncodeLaunch& l, const ClusterShape& shape, cudaStream_t stream) {
    EncodeArgs args{l.units, l.maps, l.num_units, l.relative ? 1u : 0u,
                    l.sizes, l.bounds, l.status, shift_mul(),
                    l.test_polls ? l.withhold_unit : ~0u, l.test_polls};
    cudaLaunchConfig_t cfg = {};
    const uint32_t clusters = min(min(l.num_units, shape.clusters), 65535u);
    cfg.gridDim = dim3(shape.c, clusters, 1);
    cfg.blockDim = dim3(kEncThreads, 1, 1);
    cfg.dynamicSmemBytes = Layout<T, G>::kTotal;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = shape.c;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    note_launch();
    return cudaLaunchKernelEx(&cfg, encode_kernel<T, G>, args);
}

cudaError_t launch_encode_stream(const EncodeLaunch& l, cudaStream_t stream, bool tail);
cudaError_t stream_free_slots(uint32_t busy_sms, uint32_t* slots);

// The clustered launch, and where it pays, its last round's units handed to
// the streaming encoder on the SMs no cluster holds.  `rounds` of the
// clustered encoder are ceil(units / clusters); when units % clusters of
// them would run a round alone, they run instead beside the others as one
// streaming CTA each, provided the clustered rounds that remain (at least
// 1.8 x the cluster size of them) outlast one unit in one CTA (measured on
// B200 for C2 pages: 17 rounds 83 us, one unit in one streaming CTA 66 us).
// While more than twice the cluster size of clustered rounds would remain,
// whole further rounds move to the free streaming slots as well (C5 pages,
// 512 units: 216 us against 222 us with the remainder alone moved).
template <typename T, typename G>
cudaError_t launch_encode_split(const EncodeLaunch& l, const ClusterShape& shape,
                                cudaStream_t stream) {
    if constexpr (sizeof(T) != 2) return launch_encode_g<T, G>(l, shape, stream);
    const uint32_t clusters = shape.clusters;
    uint32_t r = clusters ? l.num_units % clusters : 0u;
    uint32_t rounds = clusters ? l.num_units / clusters : 0u;
    uint32_t free_slots = 0;
    const bool split = l.whole_pages && !l.test_polls && l.encoder == 0 &&
                       r > 0 && rounds * 5 >= 9 * shape.c &&
                       stream_free_slots(shape.c * clusters, &free_slots) == cudaSuccess &&
                       r <= free_slots;
    if (!split) return launch_encode_g<T, G>(l, shape, stream);
    while (rounds > 2 * shape.c && r + clusters <= free_slots) {
        r += clusters;
        rounds -= 1;
    }
    EncodeLaunch head = l;
    head.num_units = l.num_units - r;
    cudaError_t err = launch_encode_g<T, G>(head, shape, stream);
    if (err != cudaSuccess) return err;
    EncodeLaunch tail = l;
    const uint32_t u0 = head.num_units;
    tail.units = l.units + u0;
    tail.sizes = l.sizes + u0;
    tail.bounds = l.bounds + u0;
    tail.status = l.status + u0;
    tail.num_units = r;
    return launch_encode_stream(tail, stream, true);
}

// Three 64 KB buffers per CTA where the unit fits, unless two 100 KB
// buffers let its clusters cover more SMs (large units, whose 64 KB slices
// need clusters of more than nine CTAs).
template <typename T>
cudaError_t launch_encode_t(const EncodeLaunch& l, cudaStream_t stream) {
    if (l.num_units == 0) return cudaErrorInvalidValue;
    const uint32_t nb_max = (l.max_n + kBlock - 1) / kBlock;
    const uint32_t c64 = slices_for<T, Geo64>(nb_max);
    const uint32_t c100 = slices_for<T, Geo100>(nb_max);
    if (c100 == 0) return cudaErrorInvalidValue;
    ClusterShape s64{0, 0}, s100{0, 0};
    cudaError_t err = cudaSuccess;
    if (c64) {
        err = cluster_shape<T, Geo64>(c64, &s64);
        if (err != cudaSuccess) return err;
    }
    if (!c64 || c64 > 9) {
        err = cluster_shape<T, Geo100>(c100, &s100);
        if (err != cudaSuccess) return err;
    }
    if (static_cast<uint64_t>(s100.c) * s100.clusters > static_cast<uint64_t>(s64.c) * s64.clusters)
        return launch_encode_split<T, Geo100>(l, s100, stream);
    return launch_encode_split<T, Geo64>(l, s64, stream);
}

// ---- streaming encoder: one CTA per unit ---------------------------------------
//
// For batches of whole BF16 pages (identity element map, 16-byte aligned
// elements): a CTA takes whole units (u = blockIdx.x + k * gridDim.x) and
// reads each one twice through a ring of 16 KB chunks that thread 0 keeps
// filled with bulk copies.  The first pass (from HBM) reduces the unit's
// extremes to its bound; the second (from L2, which the first pass filled)
// quantises each block, takes its rate from its own values, scans the
// chunk's block sizes, writes the rate bytes and copies the compacted payload
// out with one bulk copy per chunk.  The unit's running payload offset lives
// in one CTA: no cluster, no exchange.  Chunks of unit j's second pass
// alternate with chunks of unit j+1's first pass, so the first pass's HBM
// reads are in flight while the second pass computes; two CTAs per SM keep
// one CTA's barriers under the other's arithmetic.
//
// Every block takes the narrow quantiser, which also reports whether all of
// the block's |t| were below 2^15 (and none NaN): the truncating add then
// gives 2^23 + trunc(|t|), whose bits 15..31 are those of 2^23.  A chunk with
// any other block is redone with the exact instruction sequence for those
// blocks and written straight to global memory.

constexpr uint32_t kSBlocks = kThreads;                      // blocks per chunk
constexpr uint32_t kSElems = kSBlocks * kBlock;              // 8192 elements
constexpr uint32_t kSChunk = kSElems * 2;                    // 16 KB of BF16
constexpr uint32_t kSSlots = 5;                              // chunks in flight (two CTAs per SM)
constexpr uint32_t kSStage = kSBlocks * 64 + 16;             // compacted chunk + shift
constexpr uint32_t kSSmem = kSSlots * kSChunk + 2 * kSStage;

struct StreamArgs {
    const Unit* units;
    uint32_t num_units;
    uint32_t relative;
    uint64_t* sizes;
    float* bounds;
    uint32_t* status;
    ShiftMul mul;
    // launched as the programmatic dependent of a clustered launch (the
    // batch's remainder units): every CTA waits for that grid to complete
    // before it exits, so that work queued after this launch follows both
    uint32_t tail;
};

__device__ __forceinline__ uint32_t s_chunks(uint32_t n) { return (n + kSElems - 1) / kSElems; }

// A CTA's chunk order: all of unit 0's first pass, then unit j's second pass
// interleaved with unit j+1's first pass (second-pass chunk first), for
// j = 0, 1, ...  `cur` is the unit in its second pass, `nxt` the unit in its
// first (chunk counts 0 when absent).
struct SSeq {
    Unit cur, nxt;
    uint32_t ucur, unxt;
    uint32_t ccur, cnxt;
    uint32_t bi, ai;   // next second-pass chunk of cur, first-pass chunk of nxt
    uint32_t jn;       // position of nxt in the CTA's unit list
};

struct SElem {
    uint32_t c;
    bool second;    // second pass of cur (else first pass of nxt)
    bool shifted;   // nxt became cur just before this chunk
};

__device__ __forceinline__ void seq_load_nxt(const StreamArgs& a, SSeq& s) {
    s.unxt = blockIdx.x + s.jn * gridDim.x;
    s.cnxt = 0;
    if (s.unxt < a.num_units) {
        s.nxt = a.units[s.unxt];
        s.cnxt = s_chunks(s.nxt.n);
    }
}

__device__ __forceinline__ void seq_init(const StreamArgs& a, SSeq& s) {
    s.ccur = 0;
    s.bi = 0;
    s.ai = 0;
    s.jn = 0;
    s.ucur = ~0u;
    seq_load_nxt(a, s);
}

__device__ __forceinline__ bool seq_next(const StreamArgs& a, SSeq& s, SElem& e) {
    e.shifted = false;
    if (s.bi >= s.ccur && s.ai >= s.cnxt) {
        if (s.cnxt == 0) return false;
        s.cur = s.nxt;
        s.ucur = s.unxt;
        s.ccur = s.cnxt;
        s.bi = 0;
        s.ai = 0;
        ++s.jn;
        seq_load_nxt(a, s);
        e.shifted = true;
    }
    if (s.bi < s.ccur && (s.ai >= s.cnxt || s.bi <= s.ai)) {
        e.second = true;
        e.c = s.bi++;
    } else {
        e.second = false;
        e.c = s.ai++;
    }
    return true;
}

// Bulk copy of chunk c of `unit` (its 16-byte aligned part) into `slot`.
__device__ __forceinline__ void s_issue(const Unit& unit, uint32_t c, uint8_t* slot, uint64_t* bar) {
    const uint32_t e0 = c * kSElems, e1 = min(unit.n, e0 + kSElems);
    const uint32_t body = ((e1 - e0) * 2u) & ~15u;
    mbar_arrive_expect_tx(bar, body);
    if (body) bulk_load(slot, static_cast<const uint8_t*>(unit.elems) + e0 * 2u, body, bar);
}

// Thread 0: loads the next chunk of the producer's order into the slot it
// belongs to (chunk k of the order goes to slot k % kSSlots).
__device__ __forceinline__ void s_produce(const StreamArgs& a, SSeq& ps, uint32_t& issued,
                                          uint8_t* smem, uint64_t* full) {
    SElem e;
    if (!seq_next(a, ps, e)) return;
    const uint32_t s = issued % kSSlots;
    s_issue(e.second ? ps.cur : ps.nxt, e.c, smem + s * kSChunk, &full[s]);
    ++issued;
}

// The last chunk of a unit: the elements the bulk copy could not take (the
// last n % 8) from global memory and, with `pad`, +0 up to the end of the
// last block.  Every thread calls it; ends with a CTA barrier.
__device__ __forceinline__ void s_fill_tail(const Unit& unit, uint32_t e0, uint8_t* slot, bool pad) {
    const uint32_t n = unit.n;
    const uint32_t have = e0 + ((((n - e0) * 2u) & ~15u) >> 1);
    const uint32_t end = pad ? (n + kBlock - 1) / kBlock * kBlock : n;
    const uint16_t* src = static_cast<const uint16_t*>(unit.elems);
    uint16_t* dst = reinterpret_cast<uint16_t*>(slot);
    for (uint32_t e = have + threadIdx.x; e < end; e += kThreads)
        dst[e - e0] = e < n ? src[e] : uint16_t(0);
    __syncthreads();
}

// narrow_pair that also ORs both truncating sums into `orz`.
__device__ __forceinline__ uint32_t narrow_pair_z(float x_lo, float x_hi, uint64_t recip2,
                                                  const ShiftMul& mul, uint32_t& orz) {
    uint64_t x2, r2, t2;
    asm("mov.b64 %0, {%1, %2};" : "=l"(x2) : "f"(x_lo), "f"(x_hi));
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r2) : "l"(x2), "l"(recip2));
    asm("fma.rn.f32x2 %0, %1, %2, %3;"
        : "=l"(t2)
        : "l"(r2), "l"(0x3F8000003F800000ull), "l"(0x3F0000003F000000ull));
    float t_lo, t_hi;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(t_lo), "=f"(t_hi) : "l"(t2));
    const uint32_t z_lo = __float_as_uint(__fadd_rz(fabsf(t_lo), 8388608.0f));
    const uint32_t z_hi = __float_as_uint(__fadd_rz(fabsf(t_hi), 8388608.0f));
    orz |= z_lo | z_hi;
    const uint32_t trunc2 = __byte_perm(z_lo, z_hi, 0x5410);
    const uint32_t neg2 = prmt_sign(__float_as_uint(t_lo), __float_as_uint(t_hi), 0xffbbu);
    return trunc2 * mul.l1 + (neg2 & 0x00030003u);
}

// narrow_block (BF16) that also says whether the narrow quantiser was exact
// for every element of the block.
__device__ __forceinline__ uint32_t narrow_block_checked(const uint32_t (&w)[16], float recip,
                                                         const ShiftMul& mul, uint32_t (&A)[16],
                                                         bool& exact) {
    uint32_t orv = 0, orz = 0;
    uint64_t recip2;
    asm("mov.b64 %0, {%1, %1};" : "=l"(recip2) : "f"(recip));
#pragma unroll
    for (int k = 0; k < 16; ++k) {
        const int e = bitpos(k);
        A[k] = narrow_pair_z(elem<__nv_bfloat16>(w, e), elem<__nv_bfloat16>(w, e + 16), recip2,
                             mul, orz);
        orv |= A[k];
    }
    transpose16_mul<true, true>(A, mul);
    exact = (orz & 0xFFFF8000u) == 0x4B000000u;
    return (orv | (orv >> 16)) & 0xffffu;
}

// Exclusive scan of v over the CTA (one barrier: `scratch` alternates between
// two halves on consecutive calls), with the OR of two per-thread flags.
__device__ __forceinline__ uint32_t s_scan(uint32_t v, uint32_t flags, uint32_t* scratch,
                                           uint32_t& total, uint32_t& all_flags) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t x = v;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, x, d);
        if (lane >= d) x += y;
    }
    const uint32_t wf = __reduce_or_sync(0xffffffffu, flags);
    if (lane == 31) scratch[warp] = x | (wf << 24);   // a warp's total is below 2^24
    __syncthreads();
    uint32_t prefix = 0, sum = 0, f = 0;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
        const uint32_t sv = scratch[w];
        prefix += w < warp ? (sv & 0xFFFFFFu) : 0u;
        sum += sv & 0xFFFFFFu;
        f |= sv >> 24;
    }
    total = sum;
    all_flags = f;
    return prefix + x - v;
}

__global__ void __launch_bounds__(kThreads, 2) encode_stream_kernel(StreamArgs a) {
    using T = __nv_bfloat16;
    constexpr uint32_t BB = kBlock * 2;   // bytes per block
    enum : uint32_t { kFlagWait = 1, kFlagWide = 2 };
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t full[kSSlots];
    __shared__ uint32_t scan[2][kWarps];
    __shared__ float red_lo[kWarps], red_hi[kWarps];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int rho = (lane >> 1) & 3;
    const uint32_t sh = 8u * rho;
    uint8_t* const stage = smem + kSSlots * kSChunk;

    SSeq ps;   // thread 0: the producer's position
    uint32_t issued = 0;
    if (tid == 0) {
        for (uint32_t s = 0; s < kSSlots; ++s) mbar_init(&full[s], 1);
        fence_mbar_init();
        seq_init(a, ps);
        for (uint32_t s = 0; s < kSSlots; ++s) s_produce(a, ps, issued, smem, full);
    }
    __syncthreads();

    SSeq cs;   // every thread: the consumers' position
    seq_init(a, cs);
    uint32_t q = 0;          // chunks consumed
    uint32_t nscan = 0;      // scans done (scratch half)
    uint32_t stage_q = 0;    // staged chunks
    bool broken = false;
    // first pass of nxt
    float tlo = FLT_MAX, thi = -FLT_MAX;
    float neb = 0.0f, nrecip = 0.0f;
    // second pass of cur
    float eb = 0.0f, recip = 0.0f;
    uint32_t run = 0, bits = 0;
    bool fits = true;
    SElem e;
    while (seq_next(a, cs, e)) {
        if (e.shifted) {
            eb = neb;
            recip = nrecip;
            run = 0;
            bits = 0;
            fits = true;
            tlo = FLT_MAX;
            thi = -FLT_MAX;
        }
        const Unit& unit = e.second ? cs.cur : cs.nxt;
        const uint32_t n = unit.n, nb = (n + kBlock - 1) / kBlock;
        const uint32_t chunks = e.second ? cs.ccur : cs.cnxt;
        const uint32_t s = q % kSSlots;
        uint8_t* slot = smem + s * kSChunk;
        const bool ok = mbar_wait_bounded(&full[s], (q / kSSlots) & 1u, kWaitPolls);
        ++q;
        const bool last = e.c + 1 == chunks;
        if (last) s_fill_tail(unit, e.c * kSElems, slot, e.second);
        const uint32_t b0 = e.c * kSBlocks;
        const bool active = static_cast<uint32_t>(tid) < min(kSBlocks, nb - b0);
        const uint32_t valid = active ? min(n - (b0 + tid) * kBlock, uint32_t(kBlock)) : 0u;

        if (!e.second) {
            // -- first pass: extremes
            if (active) {
                const uint8_t* blk = slot + tid * BB;
                float lo, hi;
                if (valid == kBlock) {
                    uint32_t w[16];
                    bool nan;
                    load_block<T>(blk, rho, w);
                    block_extremes<T>(w, lo, hi, nan);
                } else {
                    lo = __int_as_float(0x7fffffff);
                    hi = lo;
                    for (uint32_t v = 0; v < valid; ++v) {
                        const float xv = elem_at<T>(blk, v);
                        lo = fminf(lo, xv);
                        hi = fmaxf(hi, xv);
                    }
                }
                tlo = fminf(tlo, lo);
                thi = fmaxf(thi, hi);
            }
            if (__syncthreads_or(!ok)) {   // also: every read of the slot is done
                broken = true;
                break;
            }
            if (tid == 0) s_produce(a, ps, issued, smem, full);
            if (last) {   // the unit's bound
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
                float lo = FLT_MAX, hi = -FLT_MAX;
#pragma unroll
                for (int w = 0; w < kWarps; ++w) {
                    lo = fminf(lo, red_lo[w]);
                    hi = fmaxf(hi, red_hi[w]);
                }
                neb = resolve_bound(unit.eb, lo, hi, a.relative != 0);
                nrecip = __fdiv_rn(0.5f, neb);
                // red_* are read before they are next written: the next
                // write follows this unit's whole second pass.
            }
            continue;
        }

        // -- second pass: rates, offsets, payload
        uint32_t w[16], A[16];
        uint32_t r = 0;
        bool wide = false;
        if (active) {
            load_block<T>(slot + tid * BB, rho, w);
            bool exact = false;
            const uint32_t orv = narrow_block_checked(w, recip, a.mul, A, exact);
            if (exact && recip <= FLT_MAX) {
                r = 32u - __clz(orv >> 1);
            } else {
                wide = true;
                uint32_t m = 0;
                for (int k = 0; k < kBlock; ++k) m |= uabs(exact_q<T>(w, k, rho, recip, valid));
                r = 32u - __clz(m);
            }
        }
        const uint32_t size = r ? 4u + 4u * r : 0u;
        // The staging buffer of this chunk is free once the bulk copy of two
        // chunks ago has read it (ordered before the writes below by the
        // scan's barrier).
        if (tid == 0) bulk_wait_read<1>();
        uint32_t total, flags;
        const uint32_t off = s_scan(size, (ok ? 0u : kFlagWait) | (wide ? kFlagWide : 0u),
                                    scan[nscan++ & 1u], total, flags);
        if (flags & kFlagWait) {
            broken = true;
            break;
        }
        if (tid == 0) s_produce(a, ps, issued, smem, full);   // every read of the slot is done
        if (fits && static_cast<uint64_t>(unit.capacity) < static_cast<uint64_t>(((n + kGroup - 1) / kGroup * (kGroup / kBlock))) + run + total) {
            fits = false;
            bits |= kErrCapacity;
        }
        if (fits) {
            const uint32_t hdr = ((n + kGroup - 1) / kGroup * (kGroup / kBlock));
            if (active) unit.stream[b0 + tid] = static_cast<uint8_t>(r);
            uint8_t* gdst = unit.stream + hdr + run;
            if (!(flags & kFlagWide)) {
                uint8_t* sb = stage + (stage_q & 1u) * kSStage;
                const uint32_t shift = static_cast<uint32_t>(reinterpret_cast<uintptr_t>(gdst) & 15u);
                if (r) {
                    uint32_t* o = reinterpret_cast<uint32_t*>(sb + shift + off);
#pragma unroll
                    for (int k = 0; k < 16; ++k)
                        if (k <= static_cast<int>(r)) o[k] = __funnelshift_l(A[k], A[k], sh);
                }
                fence_proxy_async_smem();   // the threads' stores, to the bulk copy
                __syncthreads();
                const uint32_t head = min((16u - shift) & 15u, total);
                const uint32_t body = (total - head) & ~15u;
                const uint32_t tail = total - head - body;
                const uint32_t* s32 = reinterpret_cast<const uint32_t*>(sb + shift);
                uint32_t* g32 = reinterpret_cast<uint32_t*>(gdst);
                if (static_cast<uint32_t>(tid) < head / 4) g32[tid] = s32[tid];
                if (tid >= 32 && static_cast<uint32_t>(tid - 32) < tail / 4) {
                    const uint32_t wd = (head + body) / 4 + (tid - 32);
                    g32[wd] = s32[wd];
                }
                if (tid == 0 && body) {
                    bulk_store(gdst + head, sb + shift + head, body);
                    bulk_commit();
                }
                ++stage_q;
            } else if (r) {
                uint32_t* out = reinterpret_cast<uint32_t*>(gdst + off);
                if (wide) {
                    wide_block<T>(w, rho, recip, valid, r, out);
                } else {
#pragma unroll
                    for (int k = 0; k < 16; ++k)
                        if (k <= static_cast<int>(r)) out[k] = __funnelshift_l(A[k], A[k], sh);
                }
            }
        }
        run += total;
        if (last) {
            const uint32_t hdr = ((n + kGroup - 1) / kGroup * (kGroup / kBlock));
            if (fits)
                for (uint32_t k = nb + tid; k < hdr; k += kThreads) unit.stream[k] = 0;
            if (tid == 0) {
                a.sizes[cs.ucur] = static_cast<uint64_t>(hdr) + run;
                a.bounds[cs.ucur] = eb;
                if (bits) *reinterpret_cast<volatile uint32_t*>(&a.status[cs.ucur]) = bits;
            }
        }
    }
    if (tid == 0) {
        if (broken) {
            for (uint32_t u = blockIdx.x; u < a.num_units; u += gridDim.x)
                *reinterpret_cast<volatile uint32_t*>(&a.status[u]) = kErrTimeout;
            // the copies still in flight land before the CTA leaves
            for (uint32_t k = q; k < issued; ++k)
                mbar_wait_bounded(&full[k % kSSlots], (k / kSSlots) & 1u, kWaitPolls);
        }
        bulk_wait<0>();
    }
    if (a.tail && tid == 0) asm volatile("griddepcontrol.wait;" ::: "memory");
}

// Device-wide figures of the streaming kernel, once per device: resident
// CTAs per SM and SMs.
cudaError_t stream_shape(int* per_sm, int* sms) {
    constexpr int kMaxDevices = 64;
    static std::atomic<int> cache[kMaxDevices];
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) return err;
    int v = dev >= 0 && dev < kMaxDevices ? cache[dev].load(std::memory_order_acquire) : 0;
    if (v <= 0) {
        err = cudaFuncSetAttribute(encode_stream_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   kSSmem);
        if (err != cudaSuccess) return err;
        int n = 0, p = 0;
        err = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (err != cudaSuccess) return err;
        err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&p, encode_stream_kernel, kThreads,
                                                            kSSmem);
        if (err != cudaSuccess) return err;
        v = (n << 8) | (p > 0 ? (p & 0xff) : 1);
        if (dev >= 0 && dev < kMaxDevices) cache[dev].store(v, std::memory_order_release);
    }
    *per_sm = v & 0xff;
    *sms = v >> 8;
    return cudaSuccess;
}

// Streaming CTAs that fit on the SMs that `busy_sms` clustered CTAs leave.
cudaError_t stream_free_slots(uint32_t busy_sms, uint32_t* slots) {
    int per_sm = 0, sms = 0;
    cudaError_t err = stream_shape(&per_sm, &sms);
    if (err != cudaSuccess) return err;
    *slots = static_cast<uint32_t>(sms) > busy_sms ? (sms - busy_sms) * per_sm : 0u;
    return cudaSuccess;
}

cudaError_t launch_encode_stream(const EncodeLaunch& l, cudaStream_t stream, bool tail) {
    int per_sm = 0, sms = 0;
    cudaError_t err = stream_shape(&per_sm, &sms);
    if (err != cudaSuccess) return err;
    StreamArgs args{l.units, l.num_units, l.relative ? 1u : 0u, l.sizes, l.bounds, l.status,
                    shift_mul(), tail ? 1u : 0u};
    const uint32_t grid = min(l.num_units, static_cast<uint32_t>(sms * per_sm));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid, 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = kSSmem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = tail ? 1 : 0;
    note_launch();
    return cudaLaunchKernelEx(&cfg, encode_stream_kernel, args);
}

}  // namespace

uint32_t encode_max_elements(ElemType type) {
    return type == ElemType::kBF16 ? kMaxCluster * Layout<__nv_bfloat16, Geo100>::kBlocks * kBlock
                                   : kMaxCluster * Layout<float, Geo100>::kBlocks * kBlock;
}

cudaError_t encode_prepare(ElemType type) {
    // Both geometries' kernels loaded on the current device and their
    // cluster shapes cached (setting a kernel attribute loads its code).
    ClusterShape s;
    cudaError_t e;
    if (type == ElemType::kBF16) {
        e = cluster_shape<__nv_bfloat16, Geo64>(1, &s);
        if (e == cudaSuccess) e = cluster_shape<__nv_bfloat16, Geo100>(1, &s);
    } else {
        e = cluster_shape<float, Geo64>(1, &s);
        if (e == cudaSuccess) e = cluster_shape<float, Geo100>(1, &s);
    }
    return e;
}

cudaError_t launch_encode(const EncodeLaunch& l, cudaStream_t stream) {
    const bool streamable = l.type == ElemType::kBF16 && l.whole_pages && !l.test_polls;
    if (streamable && (l.encoder == 2 || (l.encoder == 0 && l.max_n <= kStreamMaxElems)))
        return launch_encode_stream(l, stream, false);
    if (l.type == ElemType::kBF16) return launch_encode_t<__nv_bfloat16>(l, stream);
    return launch_encode_t<float>(l, stream);
}

}  // namespace ckv
