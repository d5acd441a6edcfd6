// Allocation-free variant of the batched BF16 compressor.
//
// Some callers cannot allocate device or pinned memory at the point where
// they compress: a serving engine that reserved all free HBM for its KV cache
// at start-up (any later cudaMalloc fails or evicts cache), code that must
// not trigger the device-wide synchronisation cudaFree implies, or a caller
// that owns no CUDA context state of its own.  ckv_compress_batch_fixed_bf16
// needs a context with grow-only workspaces; this entry point needs none.
//
// All of its scratch -- the unit descriptors, the copied pointer tables, the
// per-unit sizes, bounds and status words, and one built-in 32-element unit
// for the set-up call -- lives in one file-scope __device__ array of fixed
// size (kMaxUnits units, about 270 KB).  Host code cannot pass the array's
// name to a kernel (in host code it is a host-side stand-in, not a device
// address), so the device address is looked up with cudaGetSymbolAddress,
// with that device current, once per device, and cached.
//
// CUDA loads a library's modules lazily: a device's copy of the array, and
// the code of every kernel this entry point launches, are only created on
// that device at first use, which allocates device memory.  A launch may
// also grow the device's local-memory reservation.  The set-up call (batch
// 0) does all of that at a moment the caller chooses: it looks up the
// array, loads both encoder kernels (one for units of up to nine 64 KB
// slices per CTA, one for larger units), then compresses the built-in unit
// (in and out of the array itself) through every launch a real call makes.  Make it once per device at
// start-up, before the engine reserves its HBM and before any stream
// capture; later calls then allocate nothing.  A real call made first does
// the same set-up implicitly.
//
// Every call reuses the same array, so calls that overlap on the GPU (on
// different streams, or from different threads) race; the status words that
// must start at zero are cleared by every call.
#include "ckv.h"

#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>

#include "ckv_launch.h"

namespace ckv {
namespace {

constexpr size_t kMaxUnits = CKV_NOALLOC_MAX_UNITS;
constexpr int kMaxDevices = 64;

struct Scratch {
    Unit units[kMaxUnits];
    Map maps[1];
    const void* inputs[kMaxUnits];
    uint8_t* outputs[kMaxUnits];
    float eps[kMaxUnits];
    uint64_t sizes[kMaxUnits];
    float bounds[kMaxUnits];
    uint32_t status[kMaxUnits];
    uint32_t status_all;
    // the set-up call's unit: 32 BF16 zeros in, one compressed stream out
    __align__(16) uint16_t warm_in[32];
    __align__(16) uint8_t warm_out[2048];
};

static __device__ __align__(256) unsigned char g_scratch[sizeof(Scratch)];

static_assert(sizeof(size_t) == sizeof(uint64_t), "sizes are copied as 64-bit words");

// Descriptors from the copied pointer tables; clears the status words.
__global__ void fill_units(Scratch* s, uint32_t batch, uint32_t n, uint64_t capacity,
                           float error_bound, int have_eps) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i == 0) {
        Map m{};
        m.kind = kMapIdentity;
        s->maps[0] = m;
        s->status_all = 0;
    }
    if (i < batch) {
        Unit u{};
        u.elems = s->inputs[i];
        u.stream = s->outputs[i];
        u.capacity = capacity;
        u.n = n;
        u.map = 0;
        const float e = have_eps ? s->eps[i] : 0.0f;
        u.eb = e > 0.0f ? e : error_bound;
        s->units[i] = u;
        s->status[i] = 0;
    }
}

__global__ void fold_status(Scratch* s, uint32_t batch) {
    uint32_t bits = 0;
    for (uint32_t i = threadIdx.x; i < batch; i += blockDim.x) bits |= s->status[i];
    if (bits) atomicOr(&s->status_all, bits);
}

Scratch* scratch_address(int device) {
    static std::mutex lock;
    static Scratch* addr[kMaxDevices] = {};
    std::lock_guard<std::mutex> guard(lock);
    if (device < 0 || device >= kMaxDevices) return nullptr;
    if (!addr[device]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_scratch) != cudaSuccess) return nullptr;
        addr[device] = static_cast<Scratch*>(p);
    }
    return addr[device];
}

}  // namespace
}  // namespace ckv

namespace ckv {
namespace {

// One compress of `batch` units through the scratch array at `s`.
ckv_status run_noalloc(Scratch* s, const void* const* inputs, uint8_t* const* outputs,
                       const float* eps, size_t batch, size_t n, size_t capacity,
                       float error_bound, int relative, size_t* sizes, float* bounds,
                       cudaStream_t stream) {
    cudaError_t e = cudaMemcpyAsync(s->inputs, inputs, batch * sizeof(void*),
                                    cudaMemcpyHostToDevice, stream);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(s->outputs, outputs, batch * sizeof(void*), cudaMemcpyHostToDevice,
                            stream);
    if (e == cudaSuccess && eps)
        e = cudaMemcpyAsync(s->eps, eps, batch * sizeof(float), cudaMemcpyHostToDevice, stream);
    if (e != cudaSuccess) return CKV_ERR_CUDA;
    const uint32_t b = static_cast<uint32_t>(batch);
    note_launch();
    fill_units<<<(b + 255) / 256, 256, 0, stream>>>(s, b, static_cast<uint32_t>(n), capacity,
                                                    error_bound, eps ? 1 : 0);
    if (cudaGetLastError() != cudaSuccess) return CKV_ERR_CUDA;

    EncodeLaunch l{};
    l.units = s->units;
    l.maps = s->maps;
    l.num_units = b;
    l.max_n = static_cast<uint32_t>(n);
    l.relative = relative != 0;
    l.sizes = s->sizes;
    l.bounds = s->bounds;
    l.status = s->status;
    l.type = ElemType::kBF16;
    if (launch_encode(l, stream) != cudaSuccess) return CKV_ERR_CUDA;
    note_launch();
    fold_status<<<1, 256, 0, stream>>>(s, b);
    if (cudaGetLastError() != cudaSuccess) return CKV_ERR_CUDA;

    uint32_t bits = 0;
    e = cudaMemcpyAsync(sizes, s->sizes, batch * sizeof(uint64_t), cudaMemcpyDeviceToHost, stream);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(bounds, s->bounds, batch * sizeof(float), cudaMemcpyDeviceToHost,
                            stream);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(&bits, &s->status_all, sizeof(bits), cudaMemcpyDeviceToHost, stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess) return CKV_ERR_CUDA;
    if (bits & kErrCapacity) return CKV_ERR_CAPACITY;
    if (bits & kErrTimeout) return CKV_ERR_CUDA;
    if (bits) return CKV_ERR_INTERNAL;
    return CKV_OK;
}

// The set-up call: every encoder kernel loaded (units above nine 64 KB
// slices use a second one), then the built-in unit of 32 zeros through every
// launch.
ckv_status warm_up(Scratch* s, cudaStream_t stream) {
    if (encode_prepare(ElemType::kBF16) != cudaSuccess) return CKV_ERR_CUDA;
    const uint16_t zeros[32] = {};
    if (cudaMemcpyAsync(s->warm_in, zeros, sizeof(zeros), cudaMemcpyHostToDevice, stream) !=
        cudaSuccess)
        return CKV_ERR_CUDA;
    const void* in[1] = {s->warm_in};
    uint8_t* out[1] = {s->warm_out};
    size_t size = 0;
    float bound = 0.0f;
    return run_noalloc(s, in, out, nullptr, 1, 32, sizeof(s->warm_out), 1e-4f, 1, &size, &bound,
                       stream);
}

}  // namespace
}  // namespace ckv

extern "C" ckv_status ckv_compress_batch_fixed_bf16_noalloc(
    const void* const* inputs, uint8_t* const* outputs, const float* eps, size_t batch,
    size_t n, size_t capacity, float error_bound, int relative, size_t* sizes, float* bounds,
    void* stream_ptr) {
    using ckv::Scratch;
    cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
    if (batch == 0) {   // set-up call: every other argument is ignored
        int device = 0;
        if (cudaGetDevice(&device) != cudaSuccess) return CKV_ERR_CUDA;
        Scratch* s = ckv::scratch_address(device);
        if (!s) return CKV_ERR_CUDA;
        return ckv::warm_up(s, stream);
    }
    if (!inputs || !outputs || !sizes || !bounds || n == 0 || n > 0xffffffffu)
        return CKV_ERR_ARGUMENT;
    if (batch > ckv::kMaxUnits) {
        std::fprintf(stderr,
                     "ckv_compress_batch_fixed_bf16_noalloc: batch of %zu units exceeds the "
                     "fixed scratch of %zu units\n",
                     batch, ckv::kMaxUnits);
        return CKV_ERR_ARGUMENT;
    }
    if (n > ckv::encode_max_elements(ckv::ElemType::kBF16)) return CKV_ERR_UNSUPPORTED;
    if (capacity < ckv_estimate_compressed_buffer_size(n * 4)) return CKV_ERR_ARGUMENT;
    for (size_t i = 0; i < batch; ++i)
        if (!inputs[i] || !outputs[i] || (reinterpret_cast<uintptr_t>(inputs[i]) & 1u) ||
            (reinterpret_cast<uintptr_t>(outputs[i]) & 3u))
            return CKV_ERR_ARGUMENT;
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess) return CKV_ERR_CUDA;
    Scratch* s = ckv::scratch_address(device);
    if (!s) return CKV_ERR_CUDA;
    return ckv::run_noalloc(s, inputs, outputs, eps, batch, n, capacity, error_bound, relative,
                            sizes, bounds, stream);
}
