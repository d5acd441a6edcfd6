// Decoder for the fixed-mode codec (sm_100a).
//
// Persistent CTAs stream "items" of 256 blocks (8192 elements).  A CTA owns
// a contiguous range of items, so consecutive items usually belong to the
// same unit and the payload offset of the next item is the current one plus
// the current item's size; only a CTA's first item (when it starts mid-unit)
// sums the rate bytes before it.
//
// Each CTA is one producer warp and eight consumer warps around a ring of
// three slots in shared memory, with a "full" and an "empty" mbarrier per
// slot and no CTA-wide barrier in the loop:
//
//   producer warp, per item: its 256 rate bytes (copied into a small shared
//     ring by cp.async three items ahead) -> block sizes -> per-block
//     payload offsets (warp scan); once the slot is
//     empty it stores offsets, rates and the item's description in the slot
//     and starts one TMA bulk copy of the item's payload into it, completing
//     on the slot's full barrier;
//   consumer warps (one block per thread): wait for full, turn the sign word
//     and bit planes back into 32 values with a register transpose,
//     dequantise, write 16-byte stores through the element map (contiguous
//     page, one of several destinations, or layer-indexed page), arrive on
//     empty.
//
// An item whose payload does not fit a slot (many blocks of rate > 15) is
// decoded straight from global memory.
//
// Dequantisation is (float)q * eb * 2.0f rounded to BF16 as the reference
// does (cuszp_batched_fixed.cu:535-549).  For |q| < 2^15 and eb in
// [2^-100, 2^100] it is evaluated as one fused multiply-add on a
// magic-number float, fma(2^23 + |q|, 2eb, -2^23 * 2eb), which rounds exactly
// once, to the same value, as the reference's two multiplies; other blocks
// use the two multiplies.
//
// Blocks whose rate is zero are not written, as in the reference decoder
// (cuszp_batched_fixed.cu:496-623 stores only inside `if (fixed_rate)`);
// zero_fill writes (float)0 * eb * 2.0f there instead.
#include "ckv_launch.h"

#include <atomic>

namespace ckv {
namespace {

constexpr uint32_t kItemBlocks = kThreads;               // 256, one per consumer thread
constexpr int kConsumerWarps = kThreads / 32;            // 8
constexpr int kCtaThreads = kThreads + 32;               // + the producer warp
constexpr int kSlots = 3;
constexpr uint32_t kPayloadCap = kItemBlocks * 64 + 32;  // every block of rate <= 15
constexpr uint32_t kOffsAt = kPayloadCap;
constexpr uint32_t kRatesAt = kOffsAt + kItemBlocks * 4;
constexpr uint32_t kSlotBytes = (kRatesAt + kItemBlocks + 127) / 128 * 128;
constexpr uint32_t kSmem = kSlots * kSlotBytes;
constexpr uint32_t kWaitPolls = 1u << 22;
constexpr int kCtasPerSm = 3;
constexpr int kAhead = 3;                 // items whose rate bytes the producer has in flight
constexpr int kRing = kAhead + 1;

struct DecodeArgs {
    const Unit* units;
    const Map* maps;
    uint32_t num_units;
    uint32_t total_items;
    uint32_t uniform_items;   // items per unit when all units are equal, else 0
    uint32_t zero_fill;
    uint32_t* status;
    ShiftMul mul;
};

// What the consumers need of the item a slot holds.
struct SlotMeta {
    const void* elems;        // destination base of the unit
    const uint8_t* payload;   // the item's payload in global memory
    uint32_t u, b0, nbs, n;
    uint32_t map, kind;       // element map index and kind
    uint32_t flags;           // kValid, kInSlot
    uint32_t lead;            // payload byte 0 sits at slot byte `lead`
    float eb;
    uint32_t pad[3];
};
enum : uint32_t { kValid = 1, kInSlot = 2 };

__device__ __forceinline__ uint32_t block_bytes(uint32_t r) { return r ? 4 + 4 * r : 0u; }

__device__ __forceinline__ uint32_t items_of(uint32_t n) {
    return (n + kBlock * kItemBlocks - 1) / (kBlock * kItemBlocks);
}

// Values of one block in element order: exact general form.
__device__ __forceinline__ void unpack_general(const uint32_t* words, uint32_t rate, float eb,
                                               float (&f)[32]) {
    const uint32_t sign = words[0];
    uint32_t mag[32];
    // planes 0..15 and 16..31 in two 16-row transposes
#pragma unroll
    for (int half = 0; half < 2; ++half) {
        uint32_t A[16];
#pragma unroll
        for (int b = 0; b < 16; ++b) {
            const int plane = 16 * half + b;
            A[b] = plane < static_cast<int>(rate) ? words[1 + plane] : 0u;
        }
        transpose16(A);
#pragma unroll
        for (int k = 0; k < 32; ++k) {
            const uint32_t bits = k < 16 ? (A[k] & 0xffffu) : (A[k - 16] >> 16);
            if (half == 0)
                mag[k] = bits;
            else
                mag[k] |= bits << 16;
        }
    }
#pragma unroll
    for (int v = 0; v < 32; ++v) {
        const int k = bitpos(v);
        const int m = static_cast<int>(mag[k]);
        f[v] = dequantize(((sign >> k) & 1u) ? -m : m, eb);
    }
}

// Values of one block for rate <= 15 with a "safe" bound: the sign word goes
// to bit 15 of every row, so row = |q| | sign << 15.  Rows k < 16 sit in the
// low half of A[k], rows k >= 16 in the high half of A[k - 16]; the moves of
// a row into place are multiplies (FMA pipe), the masks and the sign flip
// one bit select each.
//
// `whole`: the 15 words after the sign word may be read whatever the rate (a
// block in a shared-memory slot); planes at and above the rate are then
// removed by masking the rows' magnitudes instead of zeroing the words.
template <bool whole>
__device__ __forceinline__ void unpack_fast(const uint32_t* words, uint32_t rate, float eb2,
                                            float negc, const ShiftMul& mul, float (&f)[32]) {
    uint32_t A[16];
#pragma unroll
    for (int b = 0; b < 15; ++b) A[b] = whole || b < static_cast<int>(rate) ? words[1 + b] : 0u;
    A[15] = words[0];
    const uint32_t keep = whole ? (1u << rate) - 1u : 0x7fffu;
    transpose16_mul<false, true>(A, mul);
#pragma unroll
    for (int v = 0; v < 32; ++v) {
        const int k = bitpos(v);
        uint32_t mag, sign;
        if (k < 16) {
            mag = A[k];
            sign = A[k] * mul.r16;             // row bit 15 -> bit 31
        } else {
            mag = __umulhi(A[k - 16], mul.r16);   // high half -> low half
            sign = A[k - 16];
        }
        const float x = __fmaf_rn(__uint_as_float(0x4b000000u | (mag & keep)), eb2, negc);
        f[v] = __uint_as_float(__float_as_uint(x) ^ (sign & 0x80000000u));
    }
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    const __nv_bfloat162 p = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&p);
}

// A block already rounded to BF16: element 2p in the low half of w[p].
struct Bf16Words {
    uint32_t w[16];
};

// unpack_fast for BF16 output: the same values, rounded to BF16.  Two values
// share one packed fused multiply-add (fma.rn.f32x2) and one rounding
// instruction; their signs are applied to the rounded pair, since rounding
// to nearest even is symmetric (bf16(-x) == -bf16(x)): one byte permute
// brings both rows' sign bits (row bit 15) to bits 15 and 31.
template <bool whole>
__device__ __forceinline__ void unpack_fast_bf16(const uint32_t* words, uint32_t rate, float eb2,
                                                 float negc, const ShiftMul& mul, Bf16Words& out) {
    uint32_t A[16];
#pragma unroll
    for (int b = 0; b < 15; ++b) A[b] = whole || b < static_cast<int>(rate) ? words[1 + b] : 0u;
    A[15] = words[0];
    const uint32_t keep = whole ? (1u << rate) - 1u : 0x7fffu;
    transpose16_mul<false, true>(A, mul);
    uint64_t e2, c2;
    asm("mov.b64 %0, {%1, %1};" : "=l"(e2) : "f"(eb2));
    asm("mov.b64 %0, {%1, %1};" : "=l"(c2) : "f"(negc));
#pragma unroll
    for (int p = 0; p < 16; ++p) {
        const int k0 = bitpos(2 * p), k1 = bitpos(2 * p + 1);   // k1 = k0 - 1, same half
        uint32_t m0, m1, sign;
        if (k0 < 16) {
            m0 = A[k0];
            m1 = A[k1];
            sign = __byte_perm(A[k0], A[k1], 0x5010);   // bytes 1 -> bytes 1 and 3
        } else {
            m0 = __umulhi(A[k0 - 16], mul.r16);
            m1 = __umulhi(A[k1 - 16], mul.r16);
            sign = __byte_perm(A[k0 - 16], A[k1 - 16], 0x7030);   // bytes 3 -> 1 and 3
        }
        uint64_t x2, y2;
        asm("mov.b64 %0, {%1, %2};"
            : "=l"(x2)
            : "r"(0x4b000000u | (m0 & keep)), "r"(0x4b000000u | (m1 & keep)));
        asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(y2) : "l"(x2), "l"(e2), "l"(c2));
        float y0, y1;
        asm("mov.b64 {%0, %1}, %2;" : "=f"(y0), "=f"(y1) : "l"(y2));
        out.w[p] = pack_bf16x2(y0, y1) ^ (sign & 0x80008000u);
    }
}

// Value v of a block at p: from floats (rounded here) or from BF16 words.
__device__ __forceinline__ void store_elem(__nv_bfloat16* p, const float (&f)[32], int v) {
    *p = __float2bfloat16_rn(f[v]);
}
__device__ __forceinline__ void store_elem(float* p, const float (&f)[32], int v) { *p = f[v]; }
__device__ __forceinline__ void store_elem(__nv_bfloat16* p, const Bf16Words& b, int v) {
    *reinterpret_cast<uint16_t*>(p) = static_cast<uint16_t>(b.w[v >> 1] >> (16 * (v & 1)));
}

template <typename T>
__device__ __forceinline__ void store_block16(T* dst, const float (&f)[32]) {
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
}

__device__ __forceinline__ void store_block16(__nv_bfloat16* dst, const Bf16Words& b) {
    uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int c = 0; c < 4; ++c) d[c] = make_uint4(b.w[4 * c], b.w[4 * c + 1], b.w[4 * c + 2], b.w[4 * c + 3]);
}

// e / L for a run length L: a shift when L is a power of two (KV layers and
// heads), zero when e lies in the first run (one destination per page).
__device__ __forceinline__ uint32_t run_of(uint32_t e, uint32_t L) {
    if ((L & (L - 1u)) == 0u) return e >> (__ffs(L) - 1);
    return e < L ? 0u : e / L;
}

// Writes block jb of unit u (its first `valid` values) through its map.
template <typename T, typename Values>
__device__ __forceinline__ void write_block(const DecodeArgs& a, const SlotMeta& m, uint32_t jb,
                                            uint32_t valid, const Values& f) {
    const uint32_t e0 = jb * kBlock;
    if (m.kind == kMapIdentity) {
        T* dst = static_cast<T*>(const_cast<void*>(m.elems)) + e0;
        if (valid == kBlock && (reinterpret_cast<uintptr_t>(dst) & 15u) == 0) {
            store_block16(dst, f);
            return;
        }
#pragma unroll
        for (int v = 0; v < 32; ++v)
            if (static_cast<uint32_t>(v) < valid) store_elem(dst + v, f, v);
        return;
    }
    const Map map = a.maps[m.map];
    Unit unit;
    unit.elems = m.elems;
    unit.n = m.n;
    const uint32_t L = map.run;
    const uint32_t r0 = run_of(e0, L), off = e0 - r0 * L;
    T* dst = run_base<T>(unit, map, m.u, r0) + off;
    if (valid == kBlock && off + kBlock <= L && (reinterpret_cast<uintptr_t>(dst) & 15u) == 0) {
        store_block16(dst, f);
        return;
    }
#pragma unroll
    for (int v = 0; v < 32; ++v) {
        if (static_cast<uint32_t>(v) < valid) {
            const uint32_t i = e0 + v;
            const uint32_t r = run_of(i, L);
            store_elem(run_base<T>(unit, map, m.u, r) + (i - r * L), f, v);
        }
    }
}

// Item -> (unit, item index within the unit).
__device__ __forceinline__ void locate(const DecodeArgs& a, uint32_t item, uint32_t& u,
                                       uint32_t& s) {
    if (a.uniform_items) {
        u = item / a.uniform_items;
        s = item - u * a.uniform_items;
        return;
    }
    uint32_t lo = 0, hi = a.num_units;  // last unit with item0 <= item
    while (hi - lo > 1) {
        const uint32_t mid = (lo + hi) / 2;
        if (a.units[mid].item0 <= item)
            lo = mid;
        else
            hi = mid;
    }
    u = lo;
    s = item - a.units[lo].item0;
}

// The producer's view of an item: the unit's fields and this lane's 8 rate
// bytes (blocks 8*lane .. 8*lane+7 of the item, read from the rate ring).
struct PItem {
    const uint8_t* stream;
    const void* elems;
    uint64_t size;
    uint32_t u, s, b0, nbs, items, n, hdr, map, kind;
    float eb;
    uint32_t r_lo, r_hi;
};

__device__ __forceinline__ void p_open(const DecodeArgs& a, uint32_t u, uint32_t s, PItem& it) {
    const Unit unit = a.units[u];
    it.stream = unit.stream;
    it.elems = unit.elems;
    it.size = unit.capacity;
    it.u = u;
    it.n = unit.n;
    it.hdr = (unit.n + kGroup - 1) / kGroup * (kGroup / kBlock);
    it.items = items_of(unit.n);
    it.map = unit.map;
    it.kind = a.maps[unit.map].kind;
    it.eb = unit.eb;
    it.s = s;
    it.b0 = s * kItemBlocks;
    it.nbs = min(kItemBlocks, (unit.n + kBlock - 1) / kBlock - it.b0);
}

// The item after `it` in item order (its unit record loads only when the
// unit changes).
__device__ __forceinline__ void p_next(const DecodeArgs& a, const PItem& it, PItem& nx) {
    if (it.s + 1 < it.items) {
        nx = it;
        nx.s = it.s + 1;
        nx.b0 = nx.s * kItemBlocks;
        nx.nbs = min(kItemBlocks, (it.n + kBlock - 1) / kBlock - nx.b0);
    } else {
        p_open(a, it.u + 1, 0, nx);
    }
}

// Where the producer fetches rate bytes next, kAhead items ahead of the item
// it sets up.
struct RateCursor {
    const uint8_t* stream;
    uint32_t u, s, items, nb;
};

__device__ __forceinline__ void rc_open(const DecodeArgs& a, uint32_t u, uint32_t s,
                                        RateCursor& c) {
    const Unit unit = a.units[u];
    c.stream = unit.stream;
    c.u = u;
    c.s = s;
    c.items = items_of(unit.n);
    c.nb = (unit.n + kBlock - 1) / kBlock;
}

// Starts the copy of the cursor's item's rate bytes into `ring` (64 words,
// lane l copies words 2l and 2l+1; words past the unit's blocks are not
// copied and are masked where they are read), then steps the cursor.
__device__ __forceinline__ void rc_fetch(const DecodeArgs& a, RateCursor& c, uint32_t* ring) {
    const int lane = threadIdx.x & 31;
    const uint32_t b0 = c.s * kItemBlocks;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const uint32_t first = b0 + 8 * lane + 4 * h;
        // inside the header: nb <= header bytes, both multiples of 4 apart
        if (first < c.nb) cp_async4(ring + 2 * lane + h, c.stream + first);
    }
    if (c.s + 1 < c.items)
        ++c.s;
    else
        rc_open(a, c.u + 1, 0, c);
}

// This lane's 8 rate bytes of an item from the ring (blocks 8l .. 8l+7; zero
// past the item's nbs blocks).
__device__ __forceinline__ void rc_read(const uint32_t* ring, uint32_t nbs, uint32_t& lo,
                                        uint32_t& hi) {
    const int lane = threadIdx.x & 31;
    const uint32_t first = 8 * lane;
    const uint2 w = *reinterpret_cast<const uint2*>(ring + 2 * lane);
    lo = first >= nbs ? 0u : first + 4 <= nbs ? w.x : w.x & ((1u << (8 * (nbs - first))) - 1u);
    hi = first + 4 >= nbs ? 0u : first + 8 <= nbs ? w.y : w.y & ((1u << (8 * (nbs - first - 4))) - 1u);
}

template <typename T>
__global__ void __launch_bounds__(kCtaThreads, kCtasPerSm) decode_kernel(DecodeArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t full[kSlots], empty[kSlots];
    __shared__ SlotMeta meta[kSlots];
    __shared__ uint32_t red[kCtaThreads / 32][2];
    __shared__ __align__(16) uint32_t rring[kRing][kItemBlocks / 4];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

    const uint32_t begin = static_cast<uint32_t>(
        (static_cast<uint64_t>(a.total_items) * blockIdx.x) / gridDim.x);
    const uint32_t end = static_cast<uint32_t>(
        (static_cast<uint64_t>(a.total_items) * (blockIdx.x + 1)) / gridDim.x);
    if (begin >= end) return;
    if (tid == 0) {
        for (int s = 0; s < kSlots; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumerWarps);
        }
        fence_mbar_init();
    }

    // The first item's payload offset: the sizes of all blocks before it,
    // summed by the whole CTA.  The producer first starts the copies of its
    // first items' rate bytes, which need only the item's position.
    uint32_t u0, s0;
    locate(a, begin, u0, s0);
    RateCursor rc;
    if (warp == kConsumerWarps) {
        rc_open(a, u0, s0, rc);
        for (int i = 0; i < kAhead; ++i) {
            if (begin + i < end) rc_fetch(a, rc, rring[i]);
            cp_async_commit();
        }
    }
    uint64_t first_start;
    bool first_ok;
    {
        const Unit unit = a.units[u0];
        const uint32_t* words = reinterpret_cast<const uint32_t*>(unit.stream);
        const uint32_t lim = s0 * (kItemBlocks / 4);
        uint32_t acc = 0, bad = 0;
        // eight loads in flight per thread before their sums
        for (uint32_t w0 = tid; w0 < lim; w0 += 8 * kCtaThreads) {
            uint32_t x[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const uint32_t w = w0 + j * kCtaThreads;
                x[j] = w < lim ? __ldg(words + w) : 0u;
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                acc += __dp4a(x[j], 0x01010101u, 0u) + __dp4a(__vsetne4(x[j], 0u), 0x01010101u, 0u);
                bad |= __vcmpgtu4(x[j], 0x1f1f1f1fu);
            }
        }
#pragma unroll
        for (int d = 16; d > 0; d >>= 1) {
            acc += __shfl_xor_sync(0xffffffffu, acc, d);
            bad |= __shfl_xor_sync(0xffffffffu, bad, d);
        }
        if (lane == 0) {
            red[warp][0] = acc;
            red[warp][1] = bad;
        }
        __syncthreads();
        acc = 0;
        bad = 0;
#pragma unroll
        for (int w = 0; w < kCtaThreads / 32; ++w) {
            acc += red[w][0];
            bad |= red[w][1];
        }
        const uint32_t hdr = (unit.n + kGroup - 1) / kGroup * (kGroup / kBlock);
        first_start = static_cast<uint64_t>(hdr) + 4ull * acc;
        first_ok = !bad;
    }

    if (warp == kConsumerWarps) {
        // ------------------------------ producer ------------------------------
        uint32_t status = 0;
        PItem cur, nxt;
        p_open(a, u0, s0, cur);
        uint64_t start = first_start;
        bool unit_ok = first_ok;
        if (!first_ok && lane == 0) atomicOr(&a.status[cur.u], kErrBadStream);
        uint32_t k = 0;
        for (uint32_t item = begin; item < end; ++item, ++k) {
            const int slot = static_cast<int>(k % kSlots);
            const uint32_t use = k / kSlots;
            // rate bytes kAhead items ahead; this item's have landed
            if (item + kAhead < end) rc_fetch(a, rc, rring[(k + kAhead) % kRing]);
            cp_async_commit();
            cp_async_wait<kAhead>();
            rc_read(rring[k % kRing], cur.nbs, cur.r_lo, cur.r_hi);
            if (item + 1 < end) p_next(a, cur, nxt);

            // block sizes of this lane's 8 blocks, then a warp scan
            uint32_t sz[8], lane_total = 0, bad = 0;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const uint32_t r = ((j < 4 ? cur.r_lo : cur.r_hi) >> (8 * (j & 3))) & 0xffu;
                sz[j] = lane_total;
                lane_total += block_bytes(r);
                bad |= r > 31;
            }
            uint32_t x = lane_total;
#pragma unroll
            for (int d = 1; d < 32; d <<= 1) {
                const uint32_t y = __shfl_up_sync(0xffffffffu, x, d);
                if (lane >= d) x += y;
            }
            const uint32_t lane_off = x - lane_total;
            const uint32_t total = __shfl_sync(0xffffffffu, x, 31);
            bad = __any_sync(0xffffffffu, bad);
            const bool valid =
                unit_ok && !bad && cur.size >= cur.hdr && start + total <= cur.size;
            if (!valid && unit_ok && lane == 0) atomicOr(&a.status[cur.u], kErrBadStream);
            unit_ok = valid;

            const uintptr_t g0 = reinterpret_cast<uintptr_t>(cur.stream + start);
            const uintptr_t g1 = g0 + total;
            const uintptr_t limit = reinterpret_cast<uintptr_t>(cur.stream) + cur.size;
            const uint32_t lead = static_cast<uint32_t>(g0 & 15u);
            const bool in_slot = valid && lead + total + 16 <= kPayloadCap;
            // 16-byte aligned body by TMA; where rounding the end up would
            // pass the end of the stream, the words after the last 16-byte
            // boundary are copied by the lanes
            const uintptr_t ga = g0 & ~uintptr_t(15);
            const uintptr_t up = (g1 + 15) & ~uintptr_t(15);
            const uintptr_t gb = up <= limit ? up : (g1 & ~uintptr_t(15));
            const uint32_t body = in_slot && gb > ga ? static_cast<uint32_t>(gb - ga) : 0u;

            if (use > 0 && !mbar_wait_bounded(&empty[slot], (use - 1) & 1u, kWaitPolls)) {
                status |= kErrTimeout;
                break;
            }
            uint8_t* base = smem + slot * kSlotBytes;
            uint32_t* offs = reinterpret_cast<uint32_t*>(base + kOffsAt);
            reinterpret_cast<uint4*>(offs)[2 * lane] =
                make_uint4(lane_off + sz[0], lane_off + sz[1], lane_off + sz[2], lane_off + sz[3]);
            reinterpret_cast<uint4*>(offs)[2 * lane + 1] =
                make_uint4(lane_off + sz[4], lane_off + sz[5], lane_off + sz[6], lane_off + sz[7]);
            reinterpret_cast<uint2*>(base + kRatesAt)[lane] = make_uint2(cur.r_lo, cur.r_hi);
            if (in_slot)
                for (uintptr_t g = (body ? gb : g0) + 4 * lane; g < g1; g += 128)
                    *reinterpret_cast<uint32_t*>(base + (g - ga)) =
                        __ldg(reinterpret_cast<const uint32_t*>(g));
            if (lane == 0) {
                SlotMeta m;
                m.elems = cur.elems;
                m.payload = cur.stream + start;
                m.u = cur.u;
                m.b0 = cur.b0;
                m.nbs = cur.nbs;
                m.n = cur.n;
                m.map = cur.map;
                m.kind = cur.kind;
                m.flags = (valid ? kValid : 0u) | (in_slot ? kInSlot : 0u);
                m.lead = lead;
                m.eb = cur.eb;
                m.pad[0] = m.pad[1] = m.pad[2] = 0;
                meta[slot] = m;
            }
            __syncwarp();
            if (lane == 0) {
                // releases the lanes' stores above to the consumers
                mbar_arrive_expect_tx(&full[slot], body);
                if (body) bulk_load(base, reinterpret_cast<const void*>(ga), body, &full[slot]);
            }

            if (item + 1 < end) {
                if (nxt.u == cur.u) {
                    start += total;
                } else {
                    start = nxt.hdr;
                    unit_ok = true;
                }
                cur = nxt;
            }
        }
        // Every copy this warp started has landed before the CTA can exit.
        for (uint32_t j = k > kSlots ? k - kSlots : 0; j < k; ++j)
            if (!mbar_wait_bounded(&full[j % kSlots], (j / kSlots) & 1u, kWaitPolls)) {
                status |= kErrTimeout;
                break;
            }
        if (status && lane == 0) atomicOr(&a.status[0], status);
        return;
    }

    // ------------------------------ consumers ------------------------------
    uint32_t status = 0;
    const bool safe_fill = a.zero_fill != 0;
    uint32_t k = 0;
    for (uint32_t item = begin; item < end; ++item, ++k) {
        const int slot = static_cast<int>(k % kSlots);
        if (!mbar_wait_bounded(&full[slot], (k / kSlots) & 1u, kWaitPolls)) {
            status |= kErrTimeout;
            break;
        }
        const uint8_t* base = smem + slot * kSlotBytes;
        const SlotMeta m = meta[slot];
        const uint32_t off = reinterpret_cast<const uint32_t*>(base + kOffsAt)[tid];
        const uint32_t rate = base[kRatesAt + tid];
        const uint32_t bytes = block_bytes(rate);
        const bool readable = !(m.flags & kInSlot) || m.lead + off + bytes <= kPayloadCap;
        if ((m.flags & kValid) && readable && static_cast<uint32_t>(tid) < m.nbs &&
            (rate || safe_fill)) {
            const uint32_t jb = m.b0 + tid;
            const uint32_t valid = min(m.n - jb * kBlock, uint32_t(kBlock));
            const float eb = m.eb;
            float f[32];
            bool written = false;
            if (rate) {
                const uint32_t* words =
                    (m.flags & kInSlot)
                        ? reinterpret_cast<const uint32_t*>(base + m.lead + off)
                        : reinterpret_cast<const uint32_t*>(m.payload + off);
                // eb in [2^-100, 2^100]: every nonzero |q| * 2eb is a normal
                // float, so one rounding of |q| * 2eb equals the reference's
                // rounding of |q| * eb followed by an exact doubling.
                const bool safe = eb >= 7.8886091e-31f && eb <= 1.2676506e30f;
                if (rate <= 15 && safe && sizeof(T) == 2) {
                    const float eb2 = __fmul_rn(eb, 2.0f);
                    Bf16Words h;
                    // in a slot the words past the block stay inside the slot
                    // (payload cap + offsets + rates follow the payload)
                    if (m.flags & kInSlot)
                        unpack_fast_bf16<true>(words, rate, eb2, __fmul_rn(eb2, -8388608.0f), a.mul, h);
                    else
                        unpack_fast_bf16<false>(words, rate, eb2, __fmul_rn(eb2, -8388608.0f), a.mul, h);
                    if constexpr (sizeof(T) == 2) write_block<T>(a, m, jb, valid, h);
                    written = true;
                } else if (rate <= 15 && safe) {
                    const float eb2 = __fmul_rn(eb, 2.0f);
                    if (m.flags & kInSlot)
                        unpack_fast<true>(words, rate, eb2, __fmul_rn(eb2, -8388608.0f), a.mul, f);
                    else
                        unpack_fast<false>(words, rate, eb2, __fmul_rn(eb2, -8388608.0f), a.mul, f);
                } else {
                    unpack_general(words, rate, eb, f);
                }
            } else {
                const float z = dequantize(0, eb);
#pragma unroll
                for (int v = 0; v < 32; ++v) f[v] = z;
            }
            if (!written) write_block<T>(a, m, jb, valid, f);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
    }
    if (status && lane == 0) atomicOr(&a.status[0], status);
}

// SMs of the current device, once the decoder's shared-memory size is set
// on it (both done once per device and element type).
template <typename T>
cudaError_t prepare_device(int* sms) {
    constexpr int kMaxDevices = 64;
    static std::atomic<int> cache[kMaxDevices];
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) return err;
    if (dev >= 0 && dev < kMaxDevices) {
        const int v = cache[dev].load(std::memory_order_acquire);
        if (v > 0) {
            *sms = v;
            return cudaSuccess;
        }
    }
    err = cudaFuncSetAttribute(decode_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    if (err != cudaSuccess) return err;
    int count = 0;
    err = cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, dev);
    if (err != cudaSuccess) return err;
    if (count <= 0) return cudaErrorInvalidDevice;
    if (dev >= 0 && dev < kMaxDevices) cache[dev].store(count, std::memory_order_release);
    *sms = count;
    return cudaSuccess;
}

template <typename T>
cudaError_t launch_decode_t(const DecodeLaunch& l, cudaStream_t stream) {
    if (l.num_units == 0) return cudaErrorInvalidValue;
    int sms = 0;
    cudaError_t err = prepare_device<T>(&sms);
    if (err != cudaSuccess) return err;
    DecodeArgs args{l.units, l.maps, l.num_units, l.total_items, l.uniform_items,
                    l.zero_fill ? 1u : 0u, l.status, shift_mul()};
    const uint32_t ctas = static_cast<uint32_t>(sms * kCtasPerSm);
    const uint32_t grid = l.total_items < ctas ? l.total_items : ctas;
    if (grid == 0) return cudaSuccess;
    note_launch();
    decode_kernel<T><<<grid, kCtaThreads, kSmem, stream>>>(args);
    return cudaGetLastError();
}

}  // namespace

uint32_t decode_items(uint32_t n) {
    return (n + kBlock * kItemBlocks - 1) / (kBlock * kItemBlocks);
}

cudaError_t launch_decode(const DecodeLaunch& l, cudaStream_t stream) {
    if (l.type == ElemType::kBF16) return launch_decode_t<__nv_bfloat16>(l, stream);
    return launch_decode_t<float>(l, stream);
}

}  // namespace ckv
