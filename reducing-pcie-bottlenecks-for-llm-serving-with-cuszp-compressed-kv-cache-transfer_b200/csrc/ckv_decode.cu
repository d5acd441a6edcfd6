// Decoder for the fixed-mode codec (sm_100a).
//
// Persistent CTAs stream "items" of 256 blocks (8192 elements): one block per
// thread per item.  A CTA owns a contiguous range of items, so consecutive
// items usually belong to the same unit and the payload offset of the next
// item is the current one plus the current item's size; only a CTA's first
// item (when it starts mid-unit) sums the rate bytes before it.  While a CTA
// decodes item k, the TMA bulk copy of item k+1's payload is already in
// flight into the other half of a double buffer.
//
// Per item:
//   1. each thread holds its block's rate (loaded one item ahead); one CTA
//      pass computes the exclusive scan of block sizes for item k (payload
//      offsets) and the total size of item k+1;
//   2. thread 0 issues item k+1's payload copy (16-byte aligned body by TMA,
//      the sub-16-byte tail by plain word loads);
//   3. wait for item k's payload; each thread turns its sign word and bit
//      planes back into 32 values with a register transpose and writes them
//      with 16-byte stores through the element map (contiguous page, one of
//      several destinations, or layer-indexed page).
//
// Dequantisation is (float)q * eb * 2.0f rounded to BF16 as the reference
// does (cuszp_batched_fixed.cu:535-549).  For the common case (|q| < 2^15,
// eb a normal number far from overflow) it is evaluated as one fused
// multiply-add on a magic-number float, fma(2^23 + |q|, 2eb, -2^23 * 2eb),
// which rounds exactly once, to the same value, as the reference's two
// multiplies; other blocks use the two multiplies.
//
// Blocks whose rate is zero are not written, as in the reference decoder
// (cuszp_batched_fixed.cu:496-623 stores only inside `if (fixed_rate)`);
// zero_fill writes (float)0 * eb * 2.0f there instead.
#include "ckv_launch.h"

namespace ckv {
namespace {

constexpr uint32_t kItemBlocks = kThreads;                     // 256
constexpr uint32_t kBufStride = (kItemBlocks * (4 + 4 * 32) + 32 + 15) / 16 * 16;
constexpr uint32_t kSmem = 2 * kBufStride;
constexpr uint32_t kWaitPolls = 1u << 24;
constexpr int kCtasPerSm = 3;

struct DecodeArgs {
    const Unit* units;
    const Map* maps;
    uint32_t num_units;
    uint32_t total_items;
    uint32_t uniform_items;   // items per unit when all units are equal, else 0
    uint32_t zero_fill;
    uint32_t* status;
};

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
// to bit 15 of every row, so row = |q| | sign << 15.
__device__ __forceinline__ void unpack_fast(const uint32_t* words, uint32_t rate, float eb2,
                                            float negc, float (&f)[32]) {
    uint32_t A[16];
#pragma unroll
    for (int b = 0; b < 15; ++b) A[b] = b < static_cast<int>(rate) ? words[1 + b] : 0u;
    A[15] = words[0];
    transpose16(A);
#pragma unroll
    for (int v = 0; v < 32; ++v) {
        const int k = bitpos(v);
        uint32_t mag, sign;
        if (k < 16) {
            mag = A[k] & 0x7fffu;
            sign = (A[k] << 16) & 0x80000000u;
        } else {
            mag = (A[k - 16] >> 16) & 0x7fffu;
            sign = A[k - 16] & 0x80000000u;
        }
        const float x = __fmaf_rn(__uint_as_float(0x4b000000u | mag), eb2, negc);
        f[v] = __uint_as_float(__float_as_uint(x) ^ sign);
    }
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    const __nv_bfloat162 p = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&p);
}

__device__ __forceinline__ void store_elem(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }
__device__ __forceinline__ void store_elem(float* p, float v) { *p = v; }

template <typename T>
__device__ __forceinline__ void write_block(const Unit& unit, const Map& map, uint32_t u,
                                            uint32_t jb, uint32_t valid, const float (&f)[32]) {
    const uint32_t e0 = jb * kBlock;
    const uint32_t L = run_len(unit, map);
    const uint32_t r0 = e0 / L, off = e0 - r0 * L;
    T* dst = run_base<T>(unit, map, u, r0) + off;
    if (valid == kBlock && off + kBlock <= L && (reinterpret_cast<uintptr_t>(dst) & 15u) == 0) {
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

// Item -> (unit, item index within the unit).
__device__ __forceinline__ void locate(const DecodeArgs& a, uint32_t item, uint32_t& u,
                                       uint32_t& s) {
    if (a.uniform_items) {
        u = item / a.uniform_items;
        s = item - u * a.uniform_items;
        return;
    }
    uint32_t lo = 0, hi = a.num_units;  // last unit with first_item <= item
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

struct Item {
    uint32_t u, s;       // unit, item within unit
    uint32_t b0, nbs;    // first block, blocks in the item
    uint64_t start;      // payload byte offset within the unit's stream
    uint32_t total;      // payload bytes of the item
    uint32_t rate;       // this thread's block rate (0 if none)
    bool valid;
    // the unit's descriptor fields
    const uint8_t* stream;
    uint64_t size;
    uint32_t n, hdr, map, items;
    float eb;
};

// Sets up an item and starts the load of this thread's rate byte.
__device__ __forceinline__ void open_item(const DecodeArgs& a, uint32_t u, uint32_t s, Item& it) {
    const Unit unit = a.units[u];
    it.u = u;
    it.s = s;
    it.stream = unit.stream;
    it.size = unit.capacity;
    it.n = unit.n;
    it.eb = unit.eb;
    it.map = unit.map;
    it.hdr = (unit.n + kGroup - 1) / kGroup * (kGroup / kBlock);
    it.items = items_of(unit.n);
    it.b0 = s * kItemBlocks;
    const uint32_t nb = (unit.n + kBlock - 1) / kBlock;
    it.nbs = min(kItemBlocks, nb - it.b0);
    it.rate = threadIdx.x < it.nbs ? __ldg(unit.stream + it.b0 + threadIdx.x) : 0u;
}

// The item after `it` in item order (the next unit starts at its item 0).
// Within a unit the descriptor fields are carried over, so only the rate
// byte is loaded.
__device__ __forceinline__ void next_item(const DecodeArgs& a, const Item& it, Item& nx) {
    if (it.s + 1 < it.items) {
        nx = it;
        nx.s = it.s + 1;
        nx.b0 = nx.s * kItemBlocks;
        const uint32_t nb = (it.n + kBlock - 1) / kBlock;
        nx.nbs = min(kItemBlocks, nb - nx.b0);
        nx.rate = threadIdx.x < nx.nbs ? __ldg(it.stream + nx.b0 + threadIdx.x) : 0u;
    } else {
        open_item(a, it.u + 1, 0, nx);
    }
}

template <typename T>
__global__ void __launch_bounds__(kThreads, kCtasPerSm) decode_kernel(DecodeArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ uint64_t bar[2];
    __shared__ uint32_t scan_w[kWarps], next_w[kWarps], bad_w[kWarps];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

    const uint32_t begin = static_cast<uint32_t>(
        (static_cast<uint64_t>(a.total_items) * blockIdx.x) / gridDim.x);
    const uint32_t end = static_cast<uint32_t>(
        (static_cast<uint64_t>(a.total_items) * (blockIdx.x + 1)) / gridDim.x);
    if (begin >= end) return;
    if (tid == 0) {
        mbar_init(&bar[0], 1);
        mbar_init(&bar[1], 1);
        fence_mbar_init();
    }
    __syncthreads();
    uint32_t parity = 0;  // bit b: phase parity of bar[b]

    // First item: its payload offset needs the sizes of all blocks before it.
    Item cur, nxt, nn;
    {
        uint32_t u, s;
        locate(a, begin, u, s);
        open_item(a, u, s, cur);
    }
    if (begin + 1 < end) next_item(a, cur, nxt);
    {
        const uint32_t* words = reinterpret_cast<const uint32_t*>(cur.stream);
        uint32_t acc = 0, bad = 0;
        for (uint32_t w = tid; w < cur.b0 / 4; w += kThreads) {
            const uint32_t x = __ldg(words + w);
            acc += __dp4a(x, 0x01010101u, 0u) + __dp4a(__vsetne4(x, 0u), 0x01010101u, 0u);
            bad |= __vcmpgtu4(x, 0x1f1f1f1fu);
        }
        bad |= cur.rate > 31;
        uint32_t mine = block_bytes(cur.rate);
#pragma unroll
        for (int d = 16; d > 0; d >>= 1) {
            acc += __shfl_xor_sync(0xffffffffu, acc, d);
            mine += __shfl_xor_sync(0xffffffffu, mine, d);
            bad |= __shfl_xor_sync(0xffffffffu, bad, d);
        }
        if (lane == 0) {
            scan_w[warp] = acc;
            next_w[warp] = mine;
            bad_w[warp] = bad;
        }
        __syncthreads();
        uint32_t prefix = 0, total = 0;
        bad = 0;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) {
            prefix += scan_w[w];
            total += next_w[w];
            bad |= bad_w[w];
        }
        __syncthreads();
        cur.start = static_cast<uint64_t>(cur.hdr) + 4ull * prefix;
        cur.total = total;
        cur.valid = !bad && cur.size >= cur.hdr && cur.start + total <= cur.size;
        if (!cur.valid && tid == 0) atomicOr(&a.status[cur.u], kErrBadStream);
    }

    // Issue the payload copy of an item into buffer `b`.  The bulk copy is
    // rounded out to 16-byte boundaries; where rounding up the end would pass
    // the end of the unit's stream, the last few words are loaded by the
    // threads instead.
    auto issue = [&](const Item& it, int b) {
        uint8_t* buf = smem + b * kBufStride;
        const uintptr_t g0 = reinterpret_cast<uintptr_t>(it.stream + it.start);
        const uintptr_t g1 = g0 + (it.valid ? it.total : 0u);
        const uintptr_t limit = reinterpret_cast<uintptr_t>(it.stream) + it.size;
        const uintptr_t up = (g1 + 15) & ~uintptr_t(15);
        const uintptr_t ga = g0 & ~uintptr_t(15);
        const uintptr_t gb = (it.valid && up <= limit) ? up : (g1 & ~uintptr_t(15));
        const bool body = gb > ga;
        if (tid == 0) {
            mbar_arrive_expect_tx(&bar[b], body ? static_cast<uint32_t>(gb - ga) : 0u);
            if (body)
                bulk_load(buf, reinterpret_cast<const void*>(ga), static_cast<uint32_t>(gb - ga),
                          &bar[b]);
        }
        for (uintptr_t g = (body ? gb : g0) + 4 * tid; g < g1; g += 4 * kThreads)
            *reinterpret_cast<uint32_t*>(buf + (g - ga)) =
                __ldg(reinterpret_cast<const uint32_t*>(g));
    };
    static_assert(kBufStride >= kItemBlocks * (4 + 4 * 32) + 32, "payload buffer");
    issue(cur, 0);

    uint32_t status = 0;
    int b = 0;
    for (uint32_t item = begin; item < end; ++item, b ^= 1) {
        const bool has_next = item + 1 < end;
        // rate bytes two items ahead: their load overlaps this item's decode
        if (item + 2 < end) next_item(a, nxt, nn);

        // exclusive scan of this item's block sizes + total of the next item
        const uint32_t sz = block_bytes(cur.rate);
        uint32_t x = sz;
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            const uint32_t y = __shfl_up_sync(0xffffffffu, x, d);
            if (lane >= d) x += y;
        }
        const uint32_t nrate = has_next ? nxt.rate : 0u;
        uint32_t nsz = block_bytes(nrate), nbad = nrate > 31;
#pragma unroll
        for (int d = 16; d > 0; d >>= 1) {
            nsz += __shfl_xor_sync(0xffffffffu, nsz, d);
            nbad |= __shfl_xor_sync(0xffffffffu, nbad, d);
        }
        if (lane == 31) scan_w[warp] = x;
        if (lane == 0) {
            next_w[warp] = nsz;
            bad_w[warp] = nbad;
        }
        __syncthreads();
        uint32_t off = x - sz, next_total = 0;
        nbad = 0;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) {
            off += w < warp ? scan_w[w] : 0u;
            next_total += next_w[w];
            nbad |= bad_w[w];
        }
        __syncthreads();

        if (has_next) {
            nxt.start = nxt.u == cur.u ? cur.start + cur.total : static_cast<uint64_t>(nxt.hdr);
            nxt.total = next_total;
            nxt.valid = (nxt.u == cur.u ? cur.valid : true) && !nbad && nxt.size >= nxt.hdr &&
                        nxt.start + next_total <= nxt.size;
            if (!nxt.valid && tid == 0) atomicOr(&a.status[nxt.u], kErrBadStream);
            issue(nxt, b ^ 1);
        }

        // The tail words of this item's payload were stored by the threads
        // before the scan's barriers; the TMA body completes on bar[b].
        if (!mbar_wait_bounded(&bar[b], (parity >> b) & 1u, kWaitPolls)) status |= kErrTimeout;
        parity ^= 1u << b;

        if (cur.valid && tid < static_cast<int>(cur.nbs) && (cur.rate || a.zero_fill)) {
            const uint32_t jb = cur.b0 + tid;
            const uint32_t valid = min(cur.n - jb * kBlock, uint32_t(kBlock));
            const float eb = cur.eb;
            float f[32];
            if (cur.rate) {
                const uintptr_t g0 = reinterpret_cast<uintptr_t>(cur.stream + cur.start);
                const uint32_t* words = reinterpret_cast<const uint32_t*>(
                    smem + b * kBufStride + (g0 & 15u) + off);
                // eb in [2^-100, 2^100]: every nonzero |q| * 2eb is a normal
                // float, so one rounding of |q| * 2eb equals the reference's
                // rounding of |q| * eb followed by an exact doubling.
                const bool safe = eb >= 7.8886091e-31f && eb <= 1.2676506e30f;
                if (cur.rate <= 15 && safe) {
                    const float eb2 = __fmul_rn(eb, 2.0f);
                    unpack_fast(words, cur.rate, eb2, __fmul_rn(eb2, -8388608.0f), f);
                } else {
                    unpack_general(words, cur.rate, eb, f);
                }
            } else {
                const float z = dequantize(0, eb);
#pragma unroll
                for (int v = 0; v < 32; ++v) f[v] = z;
            }
            Unit unit;
            unit.elems = a.units[cur.u].elems;
            unit.n = cur.n;
            write_block<T>(unit, a.maps[cur.map], cur.u, jb, valid, f);
        }
        cur = nxt;
        nxt = nn;
    }
    if (status && tid == 0) atomicOr(&a.status[0], status);
}

int sm_count() {
    static int count = 0;
    if (!count) {
        int dev = 0;
        cudaGetDevice(&dev);
        if (cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
            count <= 0)
            count = 148;
    }
    return count;
}

template <typename T>
cudaError_t launch_decode_t(const DecodeLaunch& l, cudaStream_t stream) {
    if (l.num_units == 0) return cudaErrorInvalidValue;
    auto kernel = decode_kernel<T>;
    cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           kSmem);
    if (err != cudaSuccess) return err;
    DecodeArgs args{l.units, l.maps, l.num_units, l.total_items, l.uniform_items,
                    l.zero_fill ? 1u : 0u, l.status};
    const uint32_t ctas = static_cast<uint32_t>(sm_count() * kCtasPerSm);
    const uint32_t grid = l.total_items < ctas ? l.total_items : ctas;
    if (grid == 0) return cudaSuccess;
    note_launch();
    decode_kernel<T><<<grid, kThreads, kSmem, stream>>>(args);
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
