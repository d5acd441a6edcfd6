// Device-side building blocks of the fixed-mode KV codec for sm_100a.
//
// Bitstream (identical to the reference's batched kernels,
// integration/cuszp_wrapper/cuszp_batched_fixed.cu):
//   * a unit of n elements is cut into 32-element blocks j;
//   * header: G*1024 rate bytes, G = ceil(n / 32768), rate_j at byte j;
//   * payload, in increasing j, for rate_j > 0: a sign word then rate_j
//     bit-plane words (4 bytes each); element v of the block sits at byte
//     v/8, bit 7 - v%8 of each word.
//
// The codec works one block per thread ("lane = block"): a thread holds the
// 32 quantised values of its block in registers and turns them into bit
// planes with a register bit-matrix transpose, which costs a few integer
// operations per element instead of one warp vote per plane.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cstdint>

namespace ckv {

constexpr int kBlock = 32;         // elements per fixed-rate block
constexpr int kGroup = 32768;      // elements per 1024 header bytes
constexpr int kThreads = 256;      // threads per CTA in every kernel
constexpr int kWarps = kThreads / 32;

// Status bits a kernel ORs into the per-unit status word.
enum : uint32_t {
    kErrCapacity = 1u << 0,   // compressed unit larger than its buffer
    kErrRateCheck = 1u << 1,  // block rate from extremes != rate from values
    kErrBadStream = 1u << 2,  // decode: rate byte > 31 or payload past size
    kErrTimeout = 1u << 3,    // a bounded wait ran out
};

// Element maps: logical element i of a unit -> address in a page.
enum : uint32_t { kMapIdentity = 0, kMapLayers = 1, kMapSplit = 2 };

struct Map {
    uint32_t kind;
    uint32_t run;              // elements per contiguous run
    // kMapLayers: [prefix][selected][run] <- [prefix][layers[s]][run]
    uint32_t selected;
    uint32_t source_layers;
    const int64_t* layers;     // device
    // kMapSplit: unit u's runs are table[u * per_unit + r]
    void* const* table;        // device
    uint32_t per_unit;
    uint32_t pad;
};

// One unit of work.  Encode: elems is the source page, stream the
// compressed output (capacity bytes).  Decode: stream is the compressed
// input (capacity = its size), elems the destination page base.
struct Unit {
    const void* elems;
    uint8_t* stream;
    uint64_t capacity;
    uint32_t n;
    uint32_t map;              // index into the launch's map table
    float eb;                  // encode: requested bound; decode: absolute bound
    uint32_t item0;            // index of the unit's first work item (decode) or chunk (encode)
};

// ---------------------------------------------------------------------------
// Arithmetic that must match the reference bit for bit.

// batch_quantization (cuszp_batched_fixed.cu:10-25).  The golden bitstreams
// of the reference's kernels on sm_100a show its mul.f32 / add.f32 pair is
// rounded separately, so both carry an explicit .rn here (which also keeps
// the code generator from fusing them).
__device__ __forceinline__ int quantize(float x, float recip) {
    int q;
    asm("{\n\t"
        ".reg .f32 r, t;\n\t"
        ".reg .pred p;\n\t"
        "mul.rn.f32 r, %1, %2;\n\t"
        "setp.ge.f32 p, r, 0fBF000000;\n\t"
        "add.rn.f32 t, r, 0f3F000000;\n\t"
        "cvt.rzi.s32.f32 %0, t;\n\t"
        "@!p sub.s32 %0, %0, 1;\n\t"
        "}"
        : "=r"(q)
        : "f"(x), "f"(recip));
    return q;
}

// |q| of a quantised value; q is never INT_MIN (see the quantiser).
__device__ __forceinline__ uint32_t uabs(int q) {
    return static_cast<uint32_t>(q < 0 ? -q : q);
}

// Absolute bound from the requested one (compute_relative_bounds_bf16_kernel,
// cuszp_batched_fixed.cu:129-130).
__device__ __forceinline__ float resolve_bound(float eps, float lo, float hi,
                                              bool relative) {
    if (!relative) return eps;
    return __fmul_rn(eps, fmaxf(__fsub_rn(hi, lo), 1e-6f));
}

// Dequantiser (cuszp_batched_fixed.cu:535-538): (float)q * eb * 2.0f.
__device__ __forceinline__ float dequantize(int q, float eb) {
    return __fmul_rn(__fmul_rn(__int2float_rn(q), eb), 2.0f);
}

__device__ __forceinline__ float bf16_lo(uint32_t w) {
    return __uint_as_float(w << 16);
}
__device__ __forceinline__ float bf16_hi(uint32_t w) {
    return __uint_as_float(w & 0xffff0000u);
}

// ---------------------------------------------------------------------------
// Register bit-matrix transposes.  A[i] is row i, bit b its column b.

// Exchanges the bits of b selected by mask with the bits of a selected by
// mask << J: t marks where the two differ, and flipping those bits in both
// swaps them (t = ((a >> J) ^ b) & mask; b ^= t; a ^= t << J).  Counted on
// sm_100a, this form issues fewer instructions per swap than two bit-selects.
template <int J>
__device__ __forceinline__ void delta_swap(uint32_t& a, uint32_t& b,
                                           uint32_t mask) {
    const uint32_t t = ((a >> J) ^ b) & mask;
    b ^= t;
    a ^= t << J;
}

// The 8-bit step as two byte permutes.
__device__ __forceinline__ void swap8(uint32_t& a, uint32_t& b) {
    const uint32_t na = __byte_perm(a, b, 0x6240);
    const uint32_t nb = __byte_perm(a, b, 0x7351);
    a = na;
    b = nb;
}

// Transpose the 16x32 matrix held as A[k] = row k | row (k+16) << 16 for
// rows of at most 16 bits: afterwards A[b] holds column b (b < 16).
// The same call inverts it (columns -> rows packed the same way).
__device__ __forceinline__ void transpose16(uint32_t (&A)[16]) {
#pragma unroll
    for (int k = 0; k < 8; ++k) swap8(A[k], A[k + 8]);
#pragma unroll
    for (int k = 0; k < 16; ++k)
        if (!(k & 4)) delta_swap<4>(A[k], A[k + 4], 0x0F0F0F0Fu);
#pragma unroll
    for (int k = 0; k < 16; ++k)
        if (!(k & 2)) delta_swap<2>(A[k], A[k + 2], 0x33333333u);
#pragma unroll
    for (int k = 0; k < 16; ++k)
        if (!(k & 1)) delta_swap<1>(A[k], A[k + 1], 0x55555555u);
}

// Multipliers that stand for shifts: x << J == x * 2^J and x >> J ==
// umulhi(x, 2^(32-J)).  They reach the kernels as launch arguments, so the
// compiler cannot turn the multiplies back into shifts: an integer
// multiply-add issues to the FMA pipe, a shift to the integer ALU pipe, and
// the bit-matrix transposes are otherwise all ALU work.
struct ShiftMul {
    uint32_t l4, l2, l1;    // 2^4, 2^2, 2^1
    uint32_t r4, r2, r1;    // 2^28, 2^30, 2^31
    uint32_t r16;           // 2^16
    uint32_t neg3;          // 2^32 - 3: x * neg3 == -3x
};

inline ShiftMul shift_mul() {
    return ShiftMul{1u << 4, 1u << 2, 1u << 1, 1u << 28, 1u << 30, 1u << 31, 1u << 16, 0xFFFFFFFDu};
}

// delta_swap with the two shifts done as multiplies (lmul = 2^J,
// rmul = 2^(32-J)).  kXor: the flip form above (t << J never carries out, as
// t lies within mask), fewest instructions; otherwise two independent
// bit-selects, the shorter dependency chain.
template <int J, bool kXor>
__device__ __forceinline__ void delta_swap_mul(uint32_t& a, uint32_t& b, uint32_t mask,
                                               uint32_t lmul, uint32_t rmul) {
    if constexpr (kXor) {
        const uint32_t t = (__umulhi(a, rmul) ^ b) & mask;
        b ^= t;
        a ^= t * lmul;
    } else {
        const uint32_t hi = mask << J;
        const uint32_t na = (a & ~hi) | ((b * lmul) & hi);
        const uint32_t nb = (b & ~mask) | (__umulhi(a, rmul) & mask);
        a = na;
        b = nb;
    }
}

// transpose16 with its 4-, 2- and 1-bit steps split between the integer
// ALU and the FMA pipe (shifts as multiplies).  kXor4 / kXor21: the flip
// form for the 4-bit step / the 2- and 1-bit steps.  Measured on B200: the
// encoder, bound by instruction issue, is fastest with the flip form
// throughout; the decoder with bit-selects in the 4-bit step and flips in
// the other two (flips throughout cost it 2-3 %).
template <bool kXor4, bool kXor21>
__device__ __forceinline__ void transpose16_mul(uint32_t (&A)[16], const ShiftMul& m) {
#pragma unroll
    for (int k = 0; k < 8; ++k) swap8(A[k], A[k + 8]);
#pragma unroll
    for (int k = 0; k < 16; ++k)
        if (!(k & 4)) delta_swap_mul<4, kXor4>(A[k], A[k + 4], 0x0F0F0F0Fu, m.l4, m.r4);
#pragma unroll
    for (int k = 0; k < 16; ++k)
        if (!(k & 2)) delta_swap_mul<2, kXor21>(A[k], A[k + 2], 0x33333333u, m.l2, m.r2);
#pragma unroll
    for (int k = 0; k < 16; ++k)
        if (!(k & 1)) delta_swap_mul<1, kXor21>(A[k], A[k + 1], 0x55555555u, m.l1, m.r1);
}

// Full 32x32 transpose (rows of up to 32 bits).
__device__ __forceinline__ void transpose32(uint32_t (&A)[32]) {
#pragma unroll
    for (int k = 0; k < 16; ++k) delta_swap<16>(A[k], A[k + 16], 0x0000FFFFu);
#pragma unroll
    for (int k = 0; k < 32; ++k)
        if (!(k & 8)) swap8(A[k], A[k + 8]);
#pragma unroll
    for (int k = 0; k < 32; ++k)
        if (!(k & 4)) delta_swap<4>(A[k], A[k + 4], 0x0F0F0F0Fu);
#pragma unroll
    for (int k = 0; k < 32; ++k)
        if (!(k & 2)) delta_swap<2>(A[k], A[k + 2], 0x33333333u);
#pragma unroll
    for (int k = 0; k < 32; ++k)
        if (!(k & 1)) delta_swap<1>(A[k], A[k + 1], 0x55555555u);
}

// Register position of block element v: byte v/8, bit 7 - v%8 of a word.
__host__ __device__ constexpr int bitpos(int v) { return (v & ~7) | (7 - (v & 7)); }

// ---------------------------------------------------------------------------
// Element maps.

__device__ __forceinline__ uint32_t run_len(const Unit& unit, const Map& m) {
    return m.kind == kMapIdentity ? (unit.n ? unit.n : 1u) : m.run;
}

// First element of run r of unit u (a run is contiguous in memory).
template <typename T>
__device__ __forceinline__ T* run_base(const Unit& unit, const Map& m,
                                       uint32_t u, uint32_t r) {
    T* base = static_cast<T*>(const_cast<void*>(unit.elems));
    if (m.kind == kMapLayers) {
        const uint32_t prefix = r / m.selected;
        const uint32_t s = r - prefix * m.selected;
        return base + (static_cast<size_t>(prefix) * m.source_layers +
                       static_cast<size_t>(m.layers[s])) *
                          m.run;
    }
    if (m.kind == kMapSplit)
        return static_cast<T*>(m.table[static_cast<size_t>(u) * m.per_unit + r]);
    return base;
}

// ---------------------------------------------------------------------------
// Asynchronous copies, barriers (PTX; no cluster multicast anywhere).

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)),
                 "r"(count)
                 : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar,
                                                      uint32_t bytes) {
    asm volatile(
        "mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(
            smem_addr(bar)),
        "r"(bytes)
        : "memory");
}

// Plain arrive (release semantics at CTA scope).
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// Waits for the phase with the given parity; gives up after `limit` polls
// (each try_wait itself blocks for a bounded, hardware-defined time).
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar,
                                                  uint32_t parity,
                                                  uint32_t limit) {
    for (uint32_t i = 0; i < limit; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}

// ---- cluster-scope barriers (distributed shared memory exchanges) ----------

// Address of the same shared variable in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t cluster_addr(const void* p, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr(p)), "r"(rank));
    return r;
}

// Arrive on an mbarrier of another CTA of the cluster (address from
// cluster_addr); orders this thread's earlier stores, peer stores included.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t remote_bar) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(remote_bar)
                 : "memory");
}

// Non-blocking test (acquire at cluster scope) of the phase with the given
// parity.
__device__ __forceinline__ bool mbar_test_wait_cluster(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// Waits for the phase with the given parity of a barrier that peers of the
// cluster arrive on, polling without suspending (a suspended try_wait is
// woken late by remote arrivals); gives up after `limit` polls.
__device__ __forceinline__ bool mbar_wait_cluster_bounded(uint64_t* bar, uint32_t parity,
                                                          uint32_t limit) {
    for (uint32_t i = 0; i < limit; ++i)
        if (mbar_test_wait_cluster(bar, parity)) return true;
    return false;
}

// Asynchronous store into another CTA's shared memory that completes
// `bytes` of transaction count on that CTA's mbarrier (both addresses from
// cluster_addr).  No fence orders it after this thread's earlier writes.
__device__ __forceinline__ void st_async_f32x2(uint32_t remote, float a, float b,
                                               uint32_t remote_bar) {
    asm volatile(
        "st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.f32 [%0], {%1, %2}, [%3];" ::"r"(
            remote),
        "f"(a), "f"(b), "r"(remote_bar)
        : "memory");
}

__device__ __forceinline__ void st_async_u32(uint32_t remote, uint32_t v, uint32_t remote_bar) {
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];" ::"r"(
                     remote),
                 "r"(v), "r"(remote_bar)
                 : "memory");
}

// Non-blocking test of the phase with the given parity (acquire, CTA scope).
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// Polls a barrier that completes by transaction count from other CTAs
// without suspending; gives up after `limit` polls.
__device__ __forceinline__ bool mbar_spin_bounded(uint64_t* bar, uint32_t parity, uint32_t limit) {
    for (uint32_t i = 0; i < limit; ++i)
        if (mbar_test_wait(bar, parity)) return true;
    return false;
}

// Asynchronous 4-byte copy global -> shared memory: no register holds the
// value, so a warp can keep several of them in flight across iterations.
__device__ __forceinline__ void cp_async4(void* smem_dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_addr(smem_dst)), "l"(src)
                 : "memory");
}

__device__ __forceinline__ void cp_async_commit() {
    asm volatile("cp.async.commit_group;" ::: "memory");
}

// Waits until at most N of this thread's committed groups are pending.
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Cluster-wide barrier that does not require converged warps.
__device__ __forceinline__ void cluster_barrier() {
    asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}

// 1-D bulk copy global -> this CTA's shared memory (16-byte aligned
// addresses, size a multiple of 16), completing on `bar`.
__device__ __forceinline__ void bulk_load(void* dst, const void* src,
                                          uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes "
        "[%0], [%1], %2, [%3];" ::"r"(smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

// 1-D bulk copy shared -> global, tracked by bulk groups.
__device__ __forceinline__ void bulk_store(void* dst, const void* src,
                                           uint32_t bytes) {
    asm volatile(
        "cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst),
        "r"(smem_addr(src)), "r"(bytes)
        : "memory");
}

__device__ __forceinline__ void bulk_commit() {
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

template <int N>
__device__ __forceinline__ void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

template <int N>
__device__ __forceinline__ void bulk_wait() {
    asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

// ---------------------------------------------------------------------------
// CTA-wide helpers (kThreads threads).

// Exclusive scan of one value per thread; returns the prefix and writes the
// CTA total to *total.  `scratch` holds kWarps + 1 words.
__device__ __forceinline__ uint32_t cta_exclusive_scan(uint32_t v,
                                                       uint32_t* scratch,
                                                       uint32_t* total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t x = v;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, x, d);
        if (lane >= d) x += y;
    }
    if (lane == 31) scratch[warp] = x;
    __syncthreads();
    uint32_t warp_prefix = 0, sum = 0;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
        const uint32_t s = scratch[w];
        warp_prefix += (w < warp) ? s : 0u;
        sum += s;
    }
    *total = sum;
    __syncthreads();
    return warp_prefix + x - v;
}

__device__ __forceinline__ uint32_t cta_sum(uint32_t v, uint32_t* scratch) {
    uint32_t total;
    cta_exclusive_scan(v, scratch, &total);
    return total;
}

}  // namespace ckv
