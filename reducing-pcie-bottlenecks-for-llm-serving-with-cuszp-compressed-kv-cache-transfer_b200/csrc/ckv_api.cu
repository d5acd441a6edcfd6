// C ABI of libckv (include/ckv.h): the CuSZpWrapper surface of the
// reference (integration/cuszp_wrapper/cuszp_wrapper.cpp) on top of the
// sm_100a encode / decode kernels.
//
// Each call turns its arguments into a list of units (one per page or
// selected-layer group) plus element maps, uploads that list through a small
// ring of pinned staging slots (one H2D copy per call), and issues ONE kernel
// launch for the whole batch.  Compression results (sizes, resolved bounds,
// status) are written by the kernel into mapped pinned memory, so the call
// only has to synchronise the stream before returning them -- no per-page
// device-to-host copies as in the reference (cuszp_wrapper.cpp:523-529).
#include "ckv.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "ckv_launch.h"

namespace ckv {

static std::atomic<uint64_t> g_launches{0};
uint64_t launches_issued() { return g_launches.load(); }
void note_launch() { g_launches.fetch_add(1); }

}  // namespace ckv

using ckv::Map;
using ckv::Unit;

namespace {

// Descriptor staging slots per context.  A slot is reused once the kernel that
// read it has finished; enough of them that the calls of a store and a
// restore in flight together (one slot per chunk launch) never wait on each
// other.
constexpr int kSlots = 32;

struct Slot {
    uint8_t* host = nullptr;   // pinned, mapped
    uint8_t* host_dev = nullptr;   // its device-side address
    uint8_t* dev = nullptr;
    size_t cap = 0;
    cudaEvent_t done = nullptr;
    bool pending = false;
};

size_t align16(size_t x) { return (x + 15) & ~size_t(15); }

}  // namespace

struct ckv_ctx {
    ckv_config config;
    int device = 0;
    bool zero_fill = false;
    std::string err;
    Slot slots[kSlots];
    int next_slot = 0;
    // compression results, mapped pinned memory
    uint64_t* sizes = nullptr;
    float* bounds = nullptr;
    uint32_t* status = nullptr;
    size_t results_cap = 0;
    // decode status words (device), accumulated until read
    uint32_t* dec_status = nullptr;
    size_t dec_status_cap = 0;
    // optional kernel timing (encode, decode, pack, INT8 encode, INT8 decode,
    // raw page copy)
    static constexpr int kTimedKinds = 6;
    bool timing = false;
    cudaEvent_t t_start[kTimedKinds] = {};
    cudaEvent_t t_stop[kTimedKinds] = {};
    bool t_valid[kTimedKinds] = {};
    // completion of a compress call's kernels (polled, see wait_stream)
    cudaEvent_t sync_ev = nullptr;
    // failure-path test hook for the next encode launch (0 polls: off)
    uint32_t test_withhold = 0;
    uint32_t test_polls = 0;
    int encoder = CKV_ENCODER_AUTO;
    // units of the last compress call (their status words stay readable)
    size_t last_units = 0;
};

namespace {

ckv_status fail(ckv_ctx* ctx, ckv_status code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    if (ctx) ctx->err = buf;
    return code;
}

ckv_status cuda_fail(ckv_ctx* ctx, const char* what, cudaError_t e) {
    return fail(ctx, CKV_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

bool fixed_1d_float(const ckv_config& c) {
    return c.processing_dim == CKV_DIM_1D && c.data_type == CKV_TYPE_FLOAT &&
           c.encoding_mode == CKV_MODE_FIXED;
}

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

// Descriptor list built on the host for one launch.
struct Batch {
    std::vector<Unit> units;
    std::vector<Map> maps;
    std::vector<void*> table;   // split-map destinations
    uint32_t max_n = 0;
};

// Grows every staging slot to at least `need` bytes (the next power of two,
// 16 KB at least).  Freeing and allocating page-locked or device memory
// synchronises the device, so all slots grow together: a context pays that a
// few times in its life, not once per slot as a batch size first appears.
ckv_status grow_slots(ckv_ctx* ctx, size_t need) {
    size_t cap = 16384;
    while (cap < need) cap <<= 1;
    for (Slot& s : ctx->slots) {
        if (s.cap >= cap) continue;
        if (s.pending) {   // its upload may still be read
            cudaError_t e = cudaEventSynchronize(s.done);
            if (e != cudaSuccess) return cuda_fail(ctx, "waiting for a descriptor slot", e);
            s.pending = false;
        }
        cudaFreeHost(s.host);
        cudaFree(s.dev);
        s.host = nullptr;
        s.dev = nullptr;
        s.cap = 0;
        cudaError_t e = cudaHostAlloc(&s.host, cap, cudaHostAllocMapped);
        if (e == cudaSuccess) e = cudaHostGetDevicePointer(&s.host_dev, s.host, 0);
        if (e != cudaSuccess) return cuda_fail(ctx, "allocating pinned descriptors", e);
        e = cudaMalloc(&s.dev, cap);
        if (e != cudaSuccess) return cuda_fail(ctx, "allocating device descriptors", e);
        s.cap = cap;
    }
    return CKV_OK;
}

// Next staging slot with at least `need` bytes, once its previous upload
// and the kernel that read it have finished.
ckv_status acquire_slot(ckv_ctx* ctx, size_t need, Slot** out) {
    Slot& s = ctx->slots[ctx->next_slot];
    ctx->next_slot = (ctx->next_slot + 1) % kSlots;
    if (s.pending) {
        cudaError_t e = cudaEventSynchronize(s.done);
        if (e != cudaSuccess) return cuda_fail(ctx, "waiting for a descriptor slot", e);
        s.pending = false;
    }
    if (!s.done) {
        cudaError_t e = cudaEventCreateWithFlags(&s.done, cudaEventDisableTiming);
        if (e != cudaSuccess) return cuda_fail(ctx, "creating an event", e);
    }
    if (need > s.cap)
        if (ckv_status st = grow_slots(ctx, need)) return st;
    *out = &s;
    return CKV_OK;
}

// Copies the batch to the device through the next staging slot; patches
// map table pointers to their device addresses.
ckv_status upload(ckv_ctx* ctx, Batch& b, cudaStream_t stream, Slot** used,
                  const Unit** d_units, const Map** d_maps) {
    const size_t units_bytes = align16(b.units.size() * sizeof(Unit));
    const size_t maps_bytes = align16(b.maps.size() * sizeof(Map));
    const size_t table_bytes = align16(b.table.size() * sizeof(void*));
    const size_t need = units_bytes + maps_bytes + table_bytes;
    Slot* sp = nullptr;
    if (ckv_status st = acquire_slot(ctx, need, &sp)) return st;
    Slot& s = *sp;
    uint8_t* h = s.host;
    void** table_dev = reinterpret_cast<void**>(s.dev + units_bytes + maps_bytes);
    for (Map& m : b.maps)
        if (m.kind == ckv::kMapSplit)
            m.table = table_dev + reinterpret_cast<uintptr_t>(m.table);  // offset -> address
    std::memcpy(h, b.units.data(), b.units.size() * sizeof(Unit));
    std::memcpy(h + units_bytes, b.maps.data(), b.maps.size() * sizeof(Map));
    if (!b.table.empty())
        std::memcpy(h + units_bytes + maps_bytes, b.table.data(), b.table.size() * sizeof(void*));
    cudaError_t e = ckv::launch_fetch(s.host_dev, s.dev, need, stream);
    if (e != cudaSuccess) return cuda_fail(ctx, "uploading descriptors", e);
    *used = &s;
    *d_units = reinterpret_cast<const Unit*>(s.dev);
    *d_maps = reinterpret_cast<const Map*>(s.dev + units_bytes);
    return CKV_OK;
}

// Kernel timing: events recorded right around a launch when enabled.
void timing_begin(ckv_ctx* ctx, int kind, cudaStream_t stream);
void timing_end(ckv_ctx* ctx, int kind, cudaStream_t stream);

void release(Slot* s, cudaStream_t stream) {
    if (s && cudaEventRecord(s->done, stream) == cudaSuccess) s->pending = true;
}

void timing_begin(ckv_ctx* ctx, int kind, cudaStream_t stream) {
    if (!ctx->timing) return;
    if (!ctx->t_start[kind]) {
        cudaEventCreate(&ctx->t_start[kind]);
        cudaEventCreate(&ctx->t_stop[kind]);
    }
    cudaEventRecord(ctx->t_start[kind], stream);
}

void timing_end(ckv_ctx* ctx, int kind, cudaStream_t stream) {
    if (!ctx->timing) return;
    ctx->t_valid[kind] = cudaEventRecord(ctx->t_stop[kind], stream) == cudaSuccess;
}

ckv_status ensure_results(ckv_ctx* ctx, size_t count) {
    if (count <= ctx->results_cap) return CKV_OK;
    cudaFreeHost(ctx->sizes);
    cudaFreeHost(ctx->bounds);
    cudaFreeHost(ctx->status);
    ctx->sizes = nullptr;
    ctx->bounds = nullptr;
    ctx->status = nullptr;
    ctx->results_cap = 0;
    size_t cap = 256;
    while (cap < count) cap <<= 1;
    cudaError_t e = cudaHostAlloc(reinterpret_cast<void**>(&ctx->sizes), cap * sizeof(uint64_t), cudaHostAllocMapped);
    if (e == cudaSuccess) e = cudaHostAlloc(reinterpret_cast<void**>(&ctx->bounds), cap * sizeof(float), cudaHostAllocMapped);
    if (e == cudaSuccess) e = cudaHostAlloc(reinterpret_cast<void**>(&ctx->status), cap * sizeof(uint32_t), cudaHostAllocMapped);
    if (e != cudaSuccess) return cuda_fail(ctx, "allocating result buffers", e);
    ctx->results_cap = cap;
    return CKV_OK;
}

ckv_status ensure_dec_status(ckv_ctx* ctx, size_t count) {
    if (count <= ctx->dec_status_cap) return CKV_OK;
    // Keep the bits recorded so far.
    uint32_t old = 0;
    if (ctx->dec_status) {
        std::vector<uint32_t> h(ctx->dec_status_cap);
        cudaDeviceSynchronize();
        cudaMemcpy(h.data(), ctx->dec_status, h.size() * 4, cudaMemcpyDeviceToHost);
        for (uint32_t v : h) old |= v;
        cudaFree(ctx->dec_status);
        ctx->dec_status = nullptr;
    }
    size_t cap = 1024;
    while (cap < count) cap <<= 1;
    cudaError_t e = cudaMalloc(&ctx->dec_status, cap * sizeof(uint32_t));
    if (e != cudaSuccess) return cuda_fail(ctx, "allocating decode status", e);
    e = cudaMemset(ctx->dec_status, 0, cap * sizeof(uint32_t));
    if (e != cudaSuccess) return cuda_fail(ctx, "clearing decode status", e);
    if (old) cudaMemcpy(ctx->dec_status, &old, 4, cudaMemcpyHostToDevice);
    ctx->dec_status_cap = cap;
    return CKV_OK;
}

float eps_of(const ckv_ctx* ctx, const float* eps, size_t i) {
    return (eps && eps[i] > 0.0f) ? eps[i] : ctx->config.error_bound;
}

ckv_status status_to_code(ckv_ctx* ctx, uint32_t bits) {
    if (!bits) return CKV_OK;
    if (bits & ckv::kErrCapacity)
        return fail(ctx, CKV_ERR_CAPACITY, "compressed data larger than its output buffer");
    if (bits & ckv::kErrBadStream)
        return fail(ctx, CKV_ERR_STREAM, "corrupt or truncated compressed page");
    if (bits & ckv::kErrTimeout)
        return fail(ctx, CKV_ERR_CUDA, "a bounded wait in the kernel ran out");
    return fail(ctx, CKV_ERR_INTERNAL, "kernel consistency check failed (status 0x%x)", bits);
}

// Waits for the work queued on `stream` so far.  A compress call returns
// once its kernels (tens to hundreds of microseconds) are done; a blocking
// wait adds the host thread's wake-up latency to every call, so the event
// is polled for up to 2 ms before the wait blocks.
cudaError_t wait_stream(ckv_ctx* ctx, cudaStream_t stream) {
    if (!ctx->sync_ev) {
        cudaError_t e = cudaEventCreateWithFlags(&ctx->sync_ev, cudaEventDisableTiming);
        if (e != cudaSuccess) return e;
    }
    cudaError_t e = cudaEventRecord(ctx->sync_ev, stream);
    if (e != cudaSuccess) return e;
    const auto start = std::chrono::steady_clock::now();
    for (;;) {
        e = cudaEventQuery(ctx->sync_ev);
        if (e != cudaErrorNotReady) return e;
        if (std::chrono::steady_clock::now() - start > std::chrono::milliseconds(2))
            return cudaEventSynchronize(ctx->sync_ev);
    }
}

// Encode a prepared batch and return sizes / bounds on the host.
ckv_status run_encode(ckv_ctx* ctx, Batch& b, ckv::ElemType type, size_t* sizes,
                      float* bounds, void* stream_ptr) {
    cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
    if (b.max_n > ckv::encode_max_elements(type))
        return fail(ctx, CKV_ERR_UNSUPPORTED,
                    "unit of %u elements exceeds the single-pass encoder limit (%u)",
                    b.max_n, ckv::encode_max_elements(type));
    DeviceGuard guard(ctx->device);
    const size_t count = b.units.size();
    for (size_t i = 0; i < count; ++i)   // the kernels write the bitstream as 32-bit words
        if (reinterpret_cast<uintptr_t>(b.units[i].stream) & 3u)
            return fail(ctx, CKV_ERR_ARGUMENT, "compressed output %zu is not 4-byte aligned", i);
    ckv_status st = ensure_results(ctx, count);
    if (st != CKV_OK) return st;
    std::memset(ctx->status, 0, count * sizeof(uint32_t));
    Slot* slot = nullptr;
    const Unit* d_units;
    const Map* d_maps;
    st = upload(ctx, b, stream, &slot, &d_units, &d_maps);
    if (st != CKV_OK) return st;
    ckv::EncodeLaunch l{};
    l.units = d_units;
    l.maps = d_maps;
    l.num_units = static_cast<uint32_t>(count);
    l.max_n = b.max_n;
    l.relative = ctx->config.use_relative_error != 0;
    l.sizes = ctx->sizes;
    l.bounds = ctx->bounds;
    l.status = ctx->status;
    l.type = type;
    l.whole_pages = true;
    for (const Unit& u : b.units)
        if (u.n == 0 || b.maps[u.map].kind != ckv::kMapIdentity ||
            (reinterpret_cast<uintptr_t>(u.elems) & 15u)) {
            l.whole_pages = false;
            break;
        }
    l.encoder = ctx->encoder;
    l.withhold_unit = ctx->test_withhold;
    l.test_polls = ctx->test_polls;
    ctx->test_polls = 0;
    ctx->last_units = count;
    timing_begin(ctx, 0, stream);
    cudaError_t e = ckv::launch_encode(l, stream);
    timing_end(ctx, 0, stream);
    release(slot, stream);
    if (e != cudaSuccess) return cuda_fail(ctx, "encode launch", e);
    e = wait_stream(ctx, stream);
    if (e != cudaSuccess) return cuda_fail(ctx, "encode", e);
    uint32_t bits = 0;
    for (size_t i = 0; i < count; ++i) {
        bits |= ctx->status[i];
        sizes[i] = static_cast<size_t>(ctx->sizes[i]);
        bounds[i] = ctx->bounds[i];
    }
    return status_to_code(ctx, bits);
}

ckv_status run_decode(ckv_ctx* ctx, Batch& b, ckv::ElemType type, void* stream_ptr) {
    cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
    DeviceGuard guard(ctx->device);
    // Empty units decode to nothing and own no work items; the decoder walks
    // units by item order, so they are dropped here (only identity-mapped
    // batches can hold them, and those index nothing by unit).
    b.units.erase(std::remove_if(b.units.begin(), b.units.end(),
                                 [](const Unit& u) { return u.n == 0; }),
                  b.units.end());
    if (b.units.empty()) return CKV_OK;
    // The decoder reads every unit's header (its rate bytes) before it can
    // check the payload against the size: a size below the header is refused
    // here, so that no read passes the caller's buffer.
    for (size_t i = 0; i < b.units.size(); ++i) {
        const Unit& u = b.units[i];
        const uint64_t hdr = (static_cast<uint64_t>(u.n) + ckv::kGroup - 1) / ckv::kGroup *
                             (ckv::kGroup / ckv::kBlock);
        if (u.capacity < hdr)
            return fail(ctx, CKV_ERR_ARGUMENT,
                        "compressed unit %zu of %llu bytes is shorter than its %llu-byte header", i,
                        static_cast<unsigned long long>(u.capacity),
                        static_cast<unsigned long long>(hdr));
    }
    const size_t count = b.units.size();
    uint32_t items = 0;
    bool uniform = true;
    for (Unit& u : b.units) {
        u.item0 = items;
        items += ckv::decode_items(u.n);
        uniform = uniform && u.n == b.units[0].n;
    }
    ckv_status st = ensure_dec_status(ctx, count);
    if (st != CKV_OK) return st;
    Slot* slot = nullptr;
    const Unit* d_units;
    const Map* d_maps;
    st = upload(ctx, b, stream, &slot, &d_units, &d_maps);
    if (st != CKV_OK) return st;
    ckv::DecodeLaunch l{};
    l.total_items = items;
    l.uniform_items = uniform ? ckv::decode_items(b.units[0].n) : 0u;
    l.units = d_units;
    l.maps = d_maps;
    l.num_units = static_cast<uint32_t>(count);
    l.max_n = b.max_n;
    l.zero_fill = ctx->zero_fill;
    l.status = ctx->dec_status;
    l.type = type;
    timing_begin(ctx, 1, stream);
    cudaError_t e = ckv::launch_decode(l, stream);
    timing_end(ctx, 1, stream);
    release(slot, stream);
    if (e != cudaSuccess) return cuda_fail(ctx, "decode launch", e);
    return CKV_OK;
}

Map identity_map() {
    Map m{};
    m.kind = ckv::kMapIdentity;
    return m;
}

Map layers_map(const int64_t* layers, size_t selected, size_t source_layers,
               size_t elements_per_layer) {
    Map m{};
    m.kind = ckv::kMapLayers;
    m.run = static_cast<uint32_t>(elements_per_layer);
    m.selected = static_cast<uint32_t>(selected);
    m.source_layers = static_cast<uint32_t>(source_layers);
    m.layers = layers;
    return m;
}

bool fits_u32(size_t v) { return v > 0 && v <= 0xffffffffu; }

ckv_status check_ctx(ckv_ctx* ctx) {
    return ctx ? CKV_OK : CKV_ERR_ARGUMENT;
}

ckv_status check_fixed(ckv_ctx* ctx, const char* what) {
    if (!fixed_1d_float(ctx->config))
        return fail(ctx, CKV_ERR_UNSUPPORTED, "%s requires fixed-mode 1D float configuration", what);
    return CKV_OK;
}

ckv_status check_stream_ptrs(ckv_ctx* ctx, const uint8_t* const* ins, const size_t* sizes,
                             size_t batch) {
    for (size_t i = 0; i < batch; ++i) {
        if (!ins[i] || sizes[i] == 0)
            return fail(ctx, CKV_ERR_ARGUMENT, "invalid compressed page %zu", i);
        if (reinterpret_cast<uintptr_t>(ins[i]) & 3u)
            return fail(ctx, CKV_ERR_ARGUMENT, "compressed page %zu is not 4-byte aligned", i);
    }
    return CKV_OK;
}

// Shared body of the BF16 / FP32 batched compressors.
ckv_status compress_batch(ckv_ctx* ctx, const void* const* inputs, uint8_t* const* outputs,
                          const float* eps, size_t batch, size_t n, size_t capacity,
                          size_t elem_bytes, size_t* sizes, float* bounds, void* stream,
                          ckv::ElemType type) {
    if (check_ctx(ctx)) return CKV_ERR_ARGUMENT;
    ctx->err.clear();
    if (batch == 0 || !inputs || !outputs || !sizes || !bounds)
        return fail(ctx, CKV_ERR_ARGUMENT, "empty batch or null argument");
    if (ckv_status s = check_fixed(ctx, "batched compression")) return s;
    if (!fits_u32(n)) return fail(ctx, CKV_ERR_ARGUMENT, "invalid element count %zu", n);
    if (capacity < ckv_estimate_compressed_buffer_size(n * 4))
        return fail(ctx, CKV_ERR_ARGUMENT, "output capacity %zu below %zu bytes", capacity,
                    ckv_estimate_compressed_buffer_size(n * 4));
    Batch b;
    b.maps.push_back(identity_map());
    b.max_n = static_cast<uint32_t>(n);
    b.units.resize(batch);
    for (size_t i = 0; i < batch; ++i) {
        if (!inputs[i] || !outputs[i])
            return fail(ctx, CKV_ERR_ARGUMENT, "null pointer for page %zu", i);
        if (reinterpret_cast<uintptr_t>(inputs[i]) % elem_bytes)
            return fail(ctx, CKV_ERR_ARGUMENT, "misaligned input page %zu", i);
        Unit& u = b.units[i];
        u = Unit{};
        u.elems = inputs[i];
        u.stream = outputs[i];
        u.capacity = capacity;
        u.n = static_cast<uint32_t>(n);
        u.map = 0;
        u.eb = eps_of(ctx, eps, i);
    }
    return run_encode(ctx, b, type, sizes, bounds, stream);
}

}  // namespace

extern "C" {

size_t ckv_estimate_compressed_buffer_size(size_t original_bytes) {
    return original_bytes * 2;
}

size_t ckv_max_compressed_size(size_t n) {
    const size_t groups = (n + ckv::kGroup - 1) / ckv::kGroup;
    const size_t blocks = (n + ckv::kBlock - 1) / ckv::kBlock;
    return groups * (ckv::kGroup / ckv::kBlock) + blocks * (4 + 4 * 32);
}

uint64_t ckv_kernel_launches(void) { return ckv::launches_issued(); }

ckv_status ckv_create(const ckv_config* config, int device_id, ckv_ctx** out) {
    if (!config || !out) return CKV_ERR_ARGUMENT;
    *out = nullptr;
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || device_id < 0 || device_id >= count)
        return CKV_ERR_CUDA;
    ckv_ctx* ctx = new ckv_ctx();
    ctx->config = *config;
    ctx->device = device_id;
    // The reference constructor makes the device current (cuszp_wrapper.cpp:37).
    cudaSetDevice(device_id);
    *out = ctx;
    return CKV_OK;
}

void ckv_destroy(ckv_ctx* ctx) {
    if (!ctx) return;
    {
        DeviceGuard guard(ctx->device);
        for (Slot& s : ctx->slots) {
            if (s.pending) cudaEventSynchronize(s.done);
            if (s.done) cudaEventDestroy(s.done);
            cudaFreeHost(s.host);
            cudaFree(s.dev);
        }
        cudaFreeHost(ctx->sizes);
        cudaFreeHost(ctx->bounds);
        cudaFreeHost(ctx->status);
        cudaFree(ctx->dec_status);
        for (int k = 0; k < ckv_ctx::kTimedKinds; ++k) {
            if (ctx->t_start[k]) cudaEventDestroy(ctx->t_start[k]);
            if (ctx->t_stop[k]) cudaEventDestroy(ctx->t_stop[k]);
        }
        if (ctx->sync_ev) cudaEventDestroy(ctx->sync_ev);
    }
    delete ctx;
}

ckv_status ckv_get_config(const ckv_ctx* ctx, ckv_config* out) {
    if (!ctx || !out) return CKV_ERR_ARGUMENT;
    *out = ctx->config;
    return CKV_OK;
}

ckv_status ckv_update_config(ckv_ctx* ctx, const ckv_config* config) {
    if (!ctx || !config) return CKV_ERR_ARGUMENT;
    ctx->config = *config;
    return CKV_OK;
}

const char* ckv_last_error(const ckv_ctx* ctx) { return ctx ? ctx->err.c_str() : "null context"; }

ckv_status ckv_set_zero_fill(ckv_ctx* ctx, int zero_fill) {
    if (!ctx) return CKV_ERR_ARGUMENT;
    ctx->zero_fill = zero_fill != 0;
    return CKV_OK;
}

ckv_status ckv_device_status(ckv_ctx* ctx, void* stream, int reset, uint32_t* bits) {
    if (!ctx || !bits) return CKV_ERR_ARGUMENT;
    *bits = 0;
    if (!ctx->dec_status) return CKV_OK;
    DeviceGuard guard(ctx->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    std::vector<uint32_t> h(ctx->dec_status_cap);
    cudaError_t e = cudaMemcpyAsync(h.data(), ctx->dec_status, h.size() * 4,
                                    cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cuda_fail(ctx, "reading decode status", e);
    for (uint32_t v : h) *bits |= v;
    if (reset) {
        e = cudaMemsetAsync(ctx->dec_status, 0, h.size() * 4, s);
        if (e != cudaSuccess) return cuda_fail(ctx, "clearing decode status", e);
    }
    return CKV_OK;
}

ckv_status ckv_compress(ckv_ctx* ctx, const float* input, size_t n, uint8_t* out,
                        size_t capacity, float eps_override, size_t* size, float* bound,
                        void* stream) {
    if (check_ctx(ctx)) return CKV_ERR_ARGUMENT;
    ctx->err.clear();
    if (!input || !out || !size || !bound || !fits_u32(n))
        return fail(ctx, CKV_ERR_ARGUMENT, "invalid compress arguments");
    if (ctx->config.processing_dim != CKV_DIM_1D || ctx->config.data_type != CKV_TYPE_FLOAT ||
        ctx->config.encoding_mode != CKV_MODE_FIXED)
        return fail(ctx, CKV_ERR_UNSUPPORTED,
                    "only the fixed-mode 1D float codec is implemented (mode %d)",
                    ctx->config.encoding_mode);
    const float eps = eps_override > 0.0f ? eps_override : ctx->config.error_bound;
    Batch b;
    b.maps.push_back(identity_map());
    b.max_n = static_cast<uint32_t>(n);
    Unit u{};
    u.elems = input;
    u.stream = out;
    u.capacity = capacity;
    u.n = static_cast<uint32_t>(n);
    u.eb = eps;
    b.units.push_back(u);
    return run_encode(ctx, b, ckv::ElemType::kF32, size, bound, stream);
}

ckv_status ckv_compress_batch_fixed(ckv_ctx* ctx, const float* const* inputs,
                                    uint8_t* const* outputs, const float* eps, size_t batch,
                                    size_t n, size_t capacity, size_t* sizes, float* bounds,
                                    void* stream) {
    return compress_batch(ctx, reinterpret_cast<const void* const*>(inputs), outputs, eps,
                          batch, n, capacity, 4, sizes, bounds, stream, ckv::ElemType::kF32);
}

ckv_status ckv_compress_batch_fixed_bf16(ckv_ctx* ctx, const void* const* inputs,
                                         uint8_t* const* outputs, const float* eps,
                                         size_t batch, size_t n, size_t capacity,
                                         size_t* sizes, float* bounds, void* stream) {
    return compress_batch(ctx, inputs, outputs, eps, batch, n, capacity, 2, sizes, bounds,
                          stream, ckv::ElemType::kBF16);
}

ckv_status ckv_compress_batch_fixed_bf16_indexed(
    ckv_ctx* ctx, const void* const* inputs, uint8_t* const* outputs,
    const int64_t* layer_indices, size_t selected, size_t prefix_count, size_t source_layers,
    size_t elements_per_layer, const float* eps, size_t batch, size_t capacity, size_t* sizes,
    float* bounds, void* stream) {
    if (check_ctx(ctx)) return CKV_ERR_ARGUMENT;
    std::vector<size_t> caps(batch, capacity);
    const int64_t* const idx[1] = {layer_indices};
    const size_t sel[1] = {selected};
    const size_t group[1] = {batch};
    return ckv_compress_batch_fixed_bf16_indexed_groups(
        ctx, inputs, outputs, idx, sel, group, 1, prefix_count, source_layers,
        elements_per_layer, eps, batch, caps.data(), sizes, bounds, stream);
}

ckv_status ckv_compress_batch_fixed_bf16_indexed_groups(
    ckv_ctx* ctx, const void* const* inputs, uint8_t* const* outputs,
    const int64_t* const* layer_indices, const size_t* selected, const size_t* group_sizes,
    size_t groups, size_t prefix_count, size_t source_layers, size_t elements_per_layer,
    const float* eps, size_t batch, const size_t* capacities, size_t* sizes, float* bounds,
    void* stream) {
    if (check_ctx(ctx)) return CKV_ERR_ARGUMENT;
    ctx->err.clear();
    if (batch == 0 || groups == 0 || !inputs || !outputs || !layer_indices || !selected ||
        !group_sizes || !capacities || !sizes || !bounds || prefix_count == 0 ||
        source_layers == 0 || elements_per_layer == 0)
        return fail(ctx, CKV_ERR_ARGUMENT, "invalid indexed compression arguments");
    if (ckv_status s = check_fixed(ctx, "indexed compression")) return s;
    Batch b;
    size_t total = 0;
    for (size_t g = 0; g < groups; ++g) {
        if (group_sizes[g] == 0 || selected[g] == 0 || selected[g] > source_layers ||
            !layer_indices[g])
            return fail(ctx, CKV_ERR_ARGUMENT, "invalid layer group %zu", g);
        total += group_sizes[g];
    }
    if (total != batch) return fail(ctx, CKV_ERR_ARGUMENT, "group sizes do not cover the batch");
    b.units.reserve(batch);
    size_t i = 0;
    for (size_t g = 0; g < groups; ++g) {
        const size_t n = prefix_count * selected[g] * elements_per_layer;
        if (!fits_u32(n)) return fail(ctx, CKV_ERR_ARGUMENT, "group %zu too large", g);
        b.maps.push_back(layers_map(layer_indices[g], selected[g], source_layers,
                                    elements_per_layer));
        b.max_n = std::max<uint32_t>(b.max_n, static_cast<uint32_t>(n));
        for (size_t k = 0; k < group_sizes[g]; ++k, ++i) {
            if (!inputs[i] || !outputs[i])
                return fail(ctx, CKV_ERR_ARGUMENT, "null pointer for unit %zu", i);
            if (reinterpret_cast<uintptr_t>(inputs[i]) & 1u)
                return fail(ctx, CKV_ERR_ARGUMENT, "misaligned input page %zu", i);
            if (capacities[i] < ckv_estimate_compressed_buffer_size(n * 4))
                return fail(ctx, CKV_ERR_ARGUMENT, "output %zu capacity %zu below %zu bytes", i,
                            capacities[i], ckv_estimate_compressed_buffer_size(n * 4));
            Unit u{};
            u.elems = inputs[i];
            u.stream = outputs[i];
            u.capacity = capacities[i];
            u.n = static_cast<uint32_t>(n);
            u.map = static_cast<uint32_t>(g);
            u.eb = eps_of(ctx, eps, i);
            b.units.push_back(u);
        }
    }
    return run_encode(ctx, b, ckv::ElemType::kBF16, sizes, bounds, stream);
}

ckv_status ckv_decompress(ckv_ctx* ctx, const uint8_t* in, size_t size, float* out, size_t n,
                          float bound, void* stream) {
    if (check_ctx(ctx)) return CKV_ERR_ARGUMENT;
    float* outs[1] = {out};
    const uint8_t* ins[1] = {in};
    const size_t sizes[1] = {size};
    const size_t ns[1] = {n};
    const float bounds[1] = {bound};
    return ckv_decompress_batch(ctx, ins, sizes, outs, ns, bounds, 1, stream);
}

ckv_status ckv_decompress_batch(ckv_ctx* ctx, const uint8_t* const* ins, const size_t* sizes,
                                float* const* outs, const size_t* n, const float* bounds,
                                size_t batch, void* stream) {
    if (check_ctx(ctx)) return CKV_ERR_ARGUMENT;
    ctx->err.clear();
    if (batch == 0) return CKV_OK;
    if (!ins || !sizes || !outs || !n || !bounds)
        return fail(ctx, CKV_ERR_ARGUMENT, "null decompression argument");
    if (ctx->config.processing_dim != CKV_DIM_1D || ctx->config.data_type != CKV_TYPE_FLOAT ||
        ctx->config.encoding_mode != CKV_MODE_FIXED)
        return fail(ctx, CKV_ERR_UNSUPPORTED,
                    "only the fixed-mode 1D float codec is implemented (mode %d)",
                    ctx->config.encoding_mode);
    if (ckv_status s = check_stream_ptrs(ctx, ins, sizes, batch)) return s;
    Batch b;
    b.maps.push_back(identity_map());
    for (size_t i = 0; i < batch; ++i) {
        if (!outs[i] || !fits_u32(n[i]) || (reinterpret_cast<uintptr_t>(outs[i]) & 3u))
            return fail(ctx, CKV_ERR_ARGUMENT, "invalid output %zu", i);
        Unit u{};
        u.elems = outs[i];
        u.stream = const_cast<uint8_t*>(ins[i]);
        u.capacity = sizes[i];
        u.n = static_cast<uint32_t>(n[i]);
        u.eb = bounds[i];
        b.units.push_back(u);
        b.max_n = std::max<uint32_t>(b.max_n, u.n);
    }
    return run_decode(ctx, b, ckv::ElemType::kF32, stream);
}

ckv_status ckv_decompress_batch_fixed_bf16(ckv_ctx* ctx, const uint8_t* const* ins,
                                           const size_t* sizes, size_t batch, void* out,
                                           size_t out_numel, size_t n, const float* bounds,
                                           void* stream) {
    if (check_ctx(ctx)) return CKV_ERR_ARGUMENT;
    ctx->err.clear();
    if (batch == 0) return CKV_OK;
    if (!ins || !sizes || !out || !bounds || !fits_u32(n) || out_numel < batch * n)
        return fail(ctx, CKV_ERR_ARGUMENT, "invalid cuSZp fixed BF16 batch metadata");
    if (ckv_status s = check_fixed(ctx, "BF16 batch decompression")) return s;
    if (ckv_status s = check_stream_ptrs(ctx, ins, sizes, batch)) return s;
    if (reinterpret_cast<uintptr_t>(out) & 1u)
        return fail(ctx, CKV_ERR_ARGUMENT, "misaligned BF16 output");
    Batch b;
    b.maps.push_back(identity_map());
    b.max_n = static_cast<uint32_t>(n);
    for (size_t i = 0; i < batch; ++i) {
        Unit u{};
        u.elems = static_cast<uint16_t*>(out) + i * n;
        u.stream = const_cast<uint8_t*>(ins[i]);
        u.capacity = sizes[i];
        u.n = static_cast<uint32_t>(n);
        u.eb = bounds[i];
        b.units.push_back(u);
    }
    return run_decode(ctx, b, ckv::ElemType::kBF16, stream);
}

ckv_status ckv_decompress_batch_fixed_bf16_scatter(ckv_ctx* ctx, const uint8_t* const* ins,
                                                   const size_t* sizes, size_t batch,
                                                   void* const* outs, size_t out_count,
                                                   size_t n, size_t per_page,
                                                   size_t elements_per_dest,
                                                   const float* bounds, void* stream) {
    if (check_ctx(ctx)) return CKV_ERR_ARGUMENT;
    ctx->err.clear();
    if (batch == 0) return CKV_OK;
    if (!ins || !sizes || !outs || !bounds || per_page == 0 || elements_per_dest == 0 ||
        n != per_page * elements_per_dest || out_count != batch * per_page || !fits_u32(n))
        return fail(ctx, CKV_ERR_ARGUMENT, "invalid cuSZp direct-scatter metadata");
    if (ckv_status s = check_fixed(ctx, "direct scatter")) return s;
    if (ckv_status s = check_stream_ptrs(ctx, ins, sizes, batch)) return s;
    Batch b;
    Map m{};
    m.kind = ckv::kMapSplit;
    m.run = static_cast<uint32_t>(elements_per_dest);
    m.per_unit = static_cast<uint32_t>(per_page);
    m.table = nullptr;  // offset 0 in the uploaded table
    b.maps.push_back(m);
    b.table.assign(outs, outs + out_count);
    for (size_t k = 0; k < out_count; ++k)
        if (!outs[k] || (reinterpret_cast<uintptr_t>(outs[k]) & 1u))
            return fail(ctx, CKV_ERR_ARGUMENT, "invalid BF16 direct-scatter destination");
    b.max_n = static_cast<uint32_t>(n);
    for (size_t i = 0; i < batch; ++i) {
        Unit u{};
        u.elems = nullptr;
        u.stream = const_cast<uint8_t*>(ins[i]);
        u.capacity = sizes[i];
        u.n = static_cast<uint32_t>(n);
        u.eb = bounds[i];
        b.units.push_back(u);
    }
    return run_decode(ctx, b, ckv::ElemType::kBF16, stream);
}

ckv_status ckv_decompress_batch_fixed_bf16_indexed_scatter(
    ckv_ctx* ctx, const uint8_t* const* ins, const size_t* sizes, size_t batch,
    void* const* outs, const int64_t* layer_indices, size_t selected, size_t prefix_count,
    size_t source_layers, size_t elements_per_layer, const float* bounds, void* stream) {
    if (check_ctx(ctx)) return CKV_ERR_ARGUMENT;
    ctx->err.clear();
    if (batch == 0) return CKV_OK;
    if (!ins || !sizes || !outs || !bounds || !layer_indices || prefix_count == 0 ||
        source_layers == 0 || elements_per_layer == 0 || selected == 0 ||
        selected > source_layers)
        return fail(ctx, CKV_ERR_ARGUMENT, "invalid indexed scatter arguments");
    if (ckv_status s = check_fixed(ctx, "indexed scatter")) return s;
    if (ckv_status s = check_stream_ptrs(ctx, ins, sizes, batch)) return s;
    const size_t n = prefix_count * selected * elements_per_layer;
    if (!fits_u32(n)) return fail(ctx, CKV_ERR_ARGUMENT, "unit too large");
    Batch b;
    b.maps.push_back(layers_map(layer_indices, selected, source_layers, elements_per_layer));
    b.max_n = static_cast<uint32_t>(n);
    for (size_t i = 0; i < batch; ++i) {
        if (!outs[i] || (reinterpret_cast<uintptr_t>(outs[i]) & 1u))
            return fail(ctx, CKV_ERR_ARGUMENT, "invalid indexed destination %zu", i);
        Unit u{};
        u.elems = outs[i];
        u.stream = const_cast<uint8_t*>(ins[i]);
        u.capacity = sizes[i];
        u.n = static_cast<uint32_t>(n);
        u.eb = bounds[i];
        b.units.push_back(u);
    }
    return run_decode(ctx, b, ckv::ElemType::kBF16, stream);
}

ckv_status ckv_pack(ckv_ctx* ctx, const uint8_t* const* srcs, const size_t* sizes, size_t count,
                    uint8_t* dst, size_t capacity, size_t align, size_t* offsets, size_t* total,
                    void* stream_ptr) {
    if (check_ctx(ctx)) return CKV_ERR_ARGUMENT;
    ctx->err.clear();
    if (!srcs || !sizes || !dst || !offsets || !total || align < 4 || (align & (align - 1)))
        return fail(ctx, CKV_ERR_ARGUMENT, "invalid pack arguments");
    *total = 0;
    if (count == 0) return CKV_OK;
    cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
    DeviceGuard guard(ctx->device);
    Slot* slot = nullptr;
    if (ckv_status st = acquire_slot(ctx, align16(count * sizeof(ckv::PackUnit)), &slot)) return st;
    auto* units = reinterpret_cast<ckv::PackUnit*>(slot->host);
    uint64_t pos = 0, max_size = 0;
    for (size_t i = 0; i < count; ++i) {
        if (!srcs[i]) return fail(ctx, CKV_ERR_ARGUMENT, "null source %zu", i);
        pos = (pos + align - 1) & ~static_cast<uint64_t>(align - 1);
        units[i] = ckv::PackUnit{srcs[i], sizes[i], pos};
        offsets[i] = static_cast<size_t>(pos);
        pos += sizes[i];
        max_size = std::max<uint64_t>(max_size, sizes[i]);
    }
    if (pos > capacity)
        return fail(ctx, CKV_ERR_CAPACITY, "packed size %llu exceeds capacity %zu",
                    static_cast<unsigned long long>(pos), capacity);
    *total = static_cast<size_t>(pos);
    cudaError_t e = ckv::launch_fetch(slot->host_dev, slot->dev,
                                      align16(count * sizeof(ckv::PackUnit)), stream);
    if (e != cudaSuccess) return cuda_fail(ctx, "uploading pack descriptors", e);
    timing_begin(ctx, 2, stream);
    e = ckv::launch_pack(reinterpret_cast<const ckv::PackUnit*>(slot->dev),
                         static_cast<uint32_t>(count), max_size, dst, stream);
    timing_end(ctx, 2, stream);
    release(slot, stream);
    if (e != cudaSuccess) return cuda_fail(ctx, "pack launch", e);
    return CKV_OK;
}

ckv_status ckv_test_withhold_exchange(ckv_ctx* ctx, uint32_t unit, uint32_t wait_polls) {
    if (check_ctx(ctx) || wait_polls == 0) return CKV_ERR_ARGUMENT;
    ctx->test_withhold = unit;
    ctx->test_polls = wait_polls;
    return CKV_OK;
}

ckv_status ckv_set_encoder(ckv_ctx* ctx, int choice) {
    if (check_ctx(ctx) || choice < CKV_ENCODER_AUTO || choice > CKV_ENCODER_STREAM)
        return CKV_ERR_ARGUMENT;
    ctx->encoder = choice;
    return CKV_OK;
}

ckv_status ckv_unit_status(ckv_ctx* ctx, size_t count, uint32_t* out) {
    if (check_ctx(ctx) || !out || count > ctx->last_units) return CKV_ERR_ARGUMENT;
    for (size_t i = 0; i < count; ++i) out[i] = ctx->status[i];
    return CKV_OK;
}

ckv_status ckv_set_kernel_timing(ckv_ctx* ctx, int enable) {
    if (!ctx) return CKV_ERR_ARGUMENT;
    ctx->timing = enable != 0;
    return CKV_OK;
}

ckv_status ckv_kernel_time(ckv_ctx* ctx, int kind, float* ms) {
    if (!ctx || !ms || kind < 0 || kind >= ckv_ctx::kTimedKinds) return CKV_ERR_ARGUMENT;
    if (!ctx->t_valid[kind]) return fail(ctx, CKV_ERR_ARGUMENT, "no timed launch of kind %d", kind);
    DeviceGuard guard(ctx->device);
    cudaError_t e = cudaEventSynchronize(ctx->t_stop[kind]);
    if (e == cudaSuccess) e = cudaEventElapsedTime(ms, ctx->t_start[kind], ctx->t_stop[kind]);
    if (e != cudaSuccess) return cuda_fail(ctx, "reading kernel time", e);
    return CKV_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Store / restore pipeline (CompressedPageStore.put_many_packed,
// vllm_v1_compressed_offload.py:371-447; _decompress_bundles_batched,
// :1618-1711; transfer_async, :2365-2385).  The reference compresses a whole
// job, packs it with torch.cat, copies it to a fresh pinned slab and
// synchronises; on restore it copies the whole slab back before the first
// decode.  Here a job runs in chunks of pages on the pipeline's own streams:
// the device-to-host copy of chunk k overlaps the compression of chunk k+1,
// the host-to-device copy of chunk k+1 the decompression of chunk k, and a
// store and a restore issued together use both directions of the link.

struct ckv_pipe {
    ckv_ctx* ctx = nullptr;
    size_t chunk = 0;   // pages per chunk
    cudaStream_t s_enc = nullptr, s_d2h = nullptr, s_h2d = nullptr, s_dec = nullptr;
    // two of each: per-page compressed staging, packed chunk, landing chunk
    uint8_t* enc[2] = {nullptr, nullptr};
    uint8_t* packed[2] = {nullptr, nullptr};
    uint8_t* land[2] = {nullptr, nullptr};
    size_t page_cap = 0;   // staging bytes per page
    size_t land_cap = 0;   // landing bytes per buffer
    cudaEvent_t ev_packed[2] = {nullptr, nullptr}, ev_copied[2] = {nullptr, nullptr};
    cudaEvent_t ev_landed[2] = {nullptr, nullptr}, ev_decoded[2] = {nullptr, nullptr};
    bool copied_used[2] = {false, false}, decoded_used[2] = {false, false};
    // chunks staged / landed so far, over every call: consecutive chunks, also
    // of consecutive jobs, alternate between the two buffers, so a job's
    // compression overlaps the previous job's copy out (and a restore's copy
    // in the previous one's decode)
    uint64_t store_seq = 0, restore_seq = 0;
    cudaEvent_t ev_in = nullptr;
    static constexpr int kTickets = 64;
    cudaEvent_t tickets[kTickets] = {};
    // read by ckv_pipe_done / ckv_pipe_wait, which other threads may call
    std::atomic<uint64_t> next_ticket{1};
    // every ticket <= retired is complete; raised before its event is reused
    std::atomic<uint64_t> retired{0};
    std::vector<const uint8_t*> srcs;
    std::vector<size_t> local;
};

namespace {

// Largest compressed page of n elements: header plus every block at rate 32.
size_t worst_page(size_t n) {
    const size_t nb = (n + ckv::kBlock - 1) / ckv::kBlock;
    const size_t hdr = (n + ckv::kGroup - 1) / ckv::kGroup * (ckv::kGroup / ckv::kBlock);
    return align16(hdr + nb * (4 + 4 * 32));
}

// Staging for chunks of pages of at most `need` bytes each (compressed or
// stored form).
ckv_status pipe_staging(ckv_pipe* p, size_t need) {
    need = align16(need);
    if (need <= p->page_cap) return CKV_OK;
    for (int k = 0; k < 2; ++k) {
        cudaFree(p->enc[k]);
        cudaFree(p->packed[k]);
        p->enc[k] = p->packed[k] = nullptr;
    }
    p->page_cap = 0;
    for (int k = 0; k < 2; ++k) {
        cudaError_t e = cudaMalloc(&p->enc[k], need * p->chunk);
        if (e == cudaSuccess) e = cudaMalloc(&p->packed[k], need * p->chunk);
        if (e != cudaSuccess) return cuda_fail(p->ctx, "allocating pipeline staging", e);
    }
    p->page_cap = need;
    return CKV_OK;
}

ckv_status pipe_landing(ckv_pipe* p, size_t bytes) {
    if (bytes <= p->land_cap) return CKV_OK;
    for (int k = 0; k < 2; ++k) {
        cudaFree(p->land[k]);
        p->land[k] = nullptr;
    }
    p->land_cap = 0;
    const size_t cap = align16(bytes);
    for (int k = 0; k < 2; ++k) {
        cudaError_t e = cudaMalloc(&p->land[k], cap);
        if (e != cudaSuccess) return cuda_fail(p->ctx, "allocating pipeline landing", e);
    }
    p->land_cap = cap;
    return CKV_OK;
}

cudaEvent_t pipe_ticket_event(ckv_pipe* p, uint64_t ticket) {
    return p->tickets[ticket % ckv_pipe::kTickets];
}

// A ticket whose event slot a newer ticket took (or is taking) over.
// pipe_issue waited for it on the host and raised `retired` before reusing
// the slot, so its work is complete.
bool pipe_retired(const ckv_pipe* p, uint64_t ticket) {
    return ticket <= p->retired.load();
}

// Records a new ticket on `stream`.  Its slot's previous ticket (kTickets
// older) retires: the host waits for it first and marks it retired before
// the event is recorded again, so that a retired ticket never aliases newer
// work.
ckv_status pipe_issue(ckv_pipe* p, cudaStream_t stream, uint64_t* ticket) {
    const uint64_t t = p->next_ticket;
    cudaEvent_t ev = pipe_ticket_event(p, t);
    cudaError_t e = cudaEventSynchronize(ev);
    if (e != cudaSuccess) return cuda_fail(p->ctx, "retiring a pipeline ticket", e);
    if (t > ckv_pipe::kTickets) p->retired.store(t - ckv_pipe::kTickets);
    e = cudaEventRecord(ev, stream);
    if (e != cudaSuccess) return cuda_fail(p->ctx, "recording a pipeline ticket", e);
    p->next_ticket = t + 1;
    if (ticket) *ticket = t;
    return CKV_OK;
}

ckv_status pipe_after(ckv_pipe* p, uint64_t after, cudaStream_t stream) {
    if (!after) return CKV_OK;
    if (after >= p->next_ticket) return fail(p->ctx, CKV_ERR_ARGUMENT, "unknown ticket");
    if (pipe_retired(p, after)) return CKV_OK;
    cudaError_t e = cudaStreamWaitEvent(stream, pipe_ticket_event(p, after), 0);
    if (e != cudaSuccess) return cuda_fail(p->ctx, "ordering after a ticket", e);
    return CKV_OK;
}

}  // namespace

extern "C" {

ckv_status ckv_pipe_create(ckv_ctx* ctx, size_t chunk_pages, ckv_pipe** out) {
    if (check_ctx(ctx) || !out || chunk_pages == 0) return CKV_ERR_ARGUMENT;
    *out = nullptr;
    DeviceGuard guard(ctx->device);
    auto* p = new ckv_pipe();
    p->ctx = ctx;
    p->chunk = chunk_pages;
    cudaError_t e = cudaSuccess;
    for (cudaStream_t* s : {&p->s_enc, &p->s_d2h, &p->s_h2d, &p->s_dec})
        if (e == cudaSuccess) e = cudaStreamCreateWithFlags(s, cudaStreamNonBlocking);
    for (int k = 0; k < 2 && e == cudaSuccess; ++k)
        for (cudaEvent_t* ev : {&p->ev_packed[k], &p->ev_copied[k], &p->ev_landed[k], &p->ev_decoded[k]})
            if (e == cudaSuccess) e = cudaEventCreateWithFlags(ev, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&p->ev_in, cudaEventDisableTiming);
    for (int k = 0; k < ckv_pipe::kTickets && e == cudaSuccess; ++k)
        e = cudaEventCreateWithFlags(&p->tickets[k], cudaEventDisableTiming);
    if (e != cudaSuccess) {
        ckv_pipe_destroy(p);
        return cuda_fail(ctx, "creating the pipeline", e);
    }
    *out = p;
    return CKV_OK;
}

void ckv_pipe_destroy(ckv_pipe* p) {
    if (!p) return;
    DeviceGuard guard(p->ctx->device);
    for (cudaStream_t s : {p->s_enc, p->s_d2h, p->s_h2d, p->s_dec})
        if (s) cudaStreamSynchronize(s);
    for (int k = 0; k < 2; ++k) {
        cudaFree(p->enc[k]);
        cudaFree(p->packed[k]);
        cudaFree(p->land[k]);
        for (cudaEvent_t ev : {p->ev_packed[k], p->ev_copied[k], p->ev_landed[k], p->ev_decoded[k]})
            if (ev) cudaEventDestroy(ev);
    }
    if (p->ev_in) cudaEventDestroy(p->ev_in);
    for (cudaEvent_t ev : p->tickets)
        if (ev) cudaEventDestroy(ev);
    for (cudaStream_t s : {p->s_enc, p->s_d2h, p->s_h2d, p->s_dec})
        if (s) cudaStreamDestroy(s);
    delete p;
}

}  // extern "C"

namespace {

// The fixed-mode store of `count` pages, each compressed as `per_page` units
// (unit g of page i is entry i * per_page + g of offsets / sizes / bounds):
// `add(b, i, g, stream, capacity)` appends that unit to the batch, whose map
// table is `maps`.  Chunks of pages are compressed (sizes on the host),
// packed and copied into the host buffer one after another on the
// pipeline's streams.
template <typename Add>
ckv_status pipe_store_units(ckv_pipe* p, size_t count, size_t per_page,
                            const std::vector<Map>& maps, uint32_t max_n, uint8_t* host,
                            size_t capacity, size_t* offsets, size_t* sizes, float* bounds,
                            size_t* total, uint64_t after, uint64_t* ticket, cudaStream_t caller,
                            Add add) {
    ckv_ctx* ctx = p->ctx;
    *total = 0;
    if (count == 0) return pipe_issue(p, caller, ticket);
    if (ckv_status st = pipe_staging(p, per_page * worst_page(max_n))) return st;
    const size_t unit_cap = p->page_cap / per_page & ~size_t(15);
    cudaError_t e = cudaEventRecord(p->ev_in, caller);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(p->s_enc, p->ev_in, 0);
    if (e != cudaSuccess) return cuda_fail(ctx, "ordering the pipeline store", e);
    if (ckv_status st = pipe_after(p, after, p->s_d2h)) return st;
    size_t pos = 0;
    for (size_t c0 = 0; c0 < count; c0 += p->chunk) {
        const int k = static_cast<int>(p->store_seq++ & 1u);
        const size_t cnt = std::min(p->chunk, count - c0);
        const size_t units = cnt * per_page, u0 = c0 * per_page;
        // the staging of chunk c - 2 has been copied out
        if (p->copied_used[k] && (e = cudaStreamWaitEvent(p->s_enc, p->ev_copied[k], 0)))
            return cuda_fail(ctx, "ordering the pipeline store", e);
        Batch b;
        b.maps = maps;
        b.max_n = max_n;
        p->srcs.resize(units);
        for (size_t i = 0; i < cnt; ++i)
            for (size_t g = 0; g < per_page; ++g) {
                uint8_t* stream = p->enc[k] + (i * per_page + g) * unit_cap;
                if (ckv_status st = add(b, c0 + i, g, stream, unit_cap)) return st;
                p->srcs[i * per_page + g] = stream;
            }
        // compress (returns once the sizes are on the host), then pack
        if (ckv_status st = run_encode(ctx, b, ckv::ElemType::kBF16, sizes + u0, bounds + u0, p->s_enc))
            return st;
        p->local.resize(units);
        size_t ctotal = 0;
        if (ckv_status st = ckv_pack(ctx, p->srcs.data(), sizes + u0, units, p->packed[k],
                                     p->page_cap * p->chunk, 16, p->local.data(), &ctotal, p->s_enc))
            return st;
        if (pos + ctotal > capacity)
            return fail(ctx, CKV_ERR_CAPACITY, "host buffer of %zu bytes too small", capacity);
        e = cudaEventRecord(p->ev_packed[k], p->s_enc);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(p->s_d2h, p->ev_packed[k], 0);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(host + pos, p->packed[k], ctotal, cudaMemcpyDeviceToHost, p->s_d2h);
        if (e == cudaSuccess) e = cudaEventRecord(p->ev_copied[k], p->s_d2h);
        if (e != cudaSuccess) return cuda_fail(ctx, "pipeline store copy", e);
        p->copied_used[k] = true;
        for (size_t i = 0; i < units; ++i) offsets[u0 + i] = pos + p->local[i];
        pos = align16(pos + ctotal);
    }
    *total = pos;
    return pipe_issue(p, p->s_d2h, ticket);
}

// The fixed-mode restore of `count` pages stored by pipe_store_units: each
// chunk's span of the host buffer is copied into a landing buffer and its
// units decoded into the pages; `add(b, i, g, stream, size)` appends unit g
// of page i (its bytes at `stream`) to the decode batch.
template <typename Add>
ckv_status pipe_restore_units(ckv_pipe* p, const uint8_t* host, const size_t* offsets,
                              const size_t* sizes, size_t count, size_t per_page,
                              const std::vector<Map>& maps, uint32_t max_n, uint64_t after,
                              uint64_t* ticket, cudaStream_t caller, Add add) {
    ckv_ctx* ctx = p->ctx;
    if (count == 0) return pipe_issue(p, caller, ticket);
    // each chunk's units are copied as one span of the host buffer
    size_t span_max = 0;
    for (size_t c0 = 0; c0 < count; c0 += p->chunk) {
        const size_t units = std::min(p->chunk, count - c0) * per_page, u0 = c0 * per_page;
        size_t lo = SIZE_MAX, hi = 0;
        for (size_t i = u0; i < u0 + units; ++i) {
            if (sizes[i] == 0 || (offsets[i] & 3u))
                return fail(ctx, CKV_ERR_ARGUMENT, "invalid stored unit %zu", i);
            lo = std::min(lo, offsets[i]);
            hi = std::max(hi, offsets[i] + sizes[i]);
        }
        span_max = std::max(span_max, hi - (lo & ~size_t(15)));
    }
    if (ckv_status st = pipe_landing(p, span_max)) return st;
    cudaError_t e = cudaEventRecord(p->ev_in, caller);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(p->s_dec, p->ev_in, 0);
    if (e != cudaSuccess) return cuda_fail(ctx, "ordering the pipeline restore", e);
    if (ckv_status st = pipe_after(p, after, p->s_h2d)) return st;
    for (size_t c0 = 0; c0 < count; c0 += p->chunk) {
        const int k = static_cast<int>(p->restore_seq++ & 1u);
        const size_t cnt = std::min(p->chunk, count - c0);
        const size_t units = cnt * per_page, u0 = c0 * per_page;
        size_t lo = SIZE_MAX, hi = 0;
        for (size_t i = u0; i < u0 + units; ++i) {
            lo = std::min(lo, offsets[i]);
            hi = std::max(hi, offsets[i] + sizes[i]);
        }
        lo &= ~size_t(15);
        // the landing buffer of chunk c - 2 has been decoded
        if (p->decoded_used[k] && (e = cudaStreamWaitEvent(p->s_h2d, p->ev_decoded[k], 0)))
            return cuda_fail(ctx, "ordering the pipeline restore", e);
        e = cudaMemcpyAsync(p->land[k], host + lo, hi - lo, cudaMemcpyHostToDevice, p->s_h2d);
        if (e == cudaSuccess) e = cudaEventRecord(p->ev_landed[k], p->s_h2d);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(p->s_dec, p->ev_landed[k], 0);
        if (e != cudaSuccess) return cuda_fail(ctx, "pipeline restore copy", e);
        Batch b;
        b.maps = maps;
        b.max_n = max_n;
        for (size_t i = 0; i < cnt; ++i)
            for (size_t g = 0; g < per_page; ++g) {
                const size_t j = (c0 + i) * per_page + g;
                if (ckv_status st = add(b, c0 + i, g, p->land[k] + (offsets[j] - lo), sizes[j]))
                    return st;
            }
        if (ckv_status st = run_decode(ctx, b, ckv::ElemType::kBF16, p->s_dec)) return st;
        if ((e = cudaEventRecord(p->ev_decoded[k], p->s_dec)))
            return cuda_fail(ctx, "pipeline restore", e);
        p->decoded_used[k] = true;
    }
    uint64_t t = 0;
    if (ckv_status st = pipe_issue(p, p->s_dec, &t)) return st;
    // like the reference's decompress calls: asynchronous on the caller's stream
    e = cudaStreamWaitEvent(caller, pipe_ticket_event(p, t), 0);
    if (e != cudaSuccess) return cuda_fail(ctx, "joining the pipeline restore", e);
    if (ticket) *ticket = t;
    return CKV_OK;
}

// Checks a layer-group description; the largest group's element count.
ckv_status check_groups(ckv_ctx* ctx, const int64_t* const* layer_indices, const size_t* selected,
                        size_t groups, size_t prefix_count, size_t source_layers,
                        size_t elements_per_layer, std::vector<Map>& maps, uint32_t* max_n) {
    if (groups == 0 || !layer_indices || !selected || prefix_count == 0 || source_layers == 0 ||
        elements_per_layer == 0)
        return fail(ctx, CKV_ERR_ARGUMENT, "invalid layer groups");
    maps.clear();
    *max_n = 0;
    for (size_t g = 0; g < groups; ++g) {
        if (!layer_indices[g] || selected[g] == 0 || selected[g] > source_layers)
            return fail(ctx, CKV_ERR_ARGUMENT, "invalid layer group %zu", g);
        const size_t n = prefix_count * selected[g] * elements_per_layer;
        if (!fits_u32(n)) return fail(ctx, CKV_ERR_ARGUMENT, "layer group %zu too large", g);
        maps.push_back(layers_map(layer_indices[g], selected[g], source_layers, elements_per_layer));
        *max_n = std::max<uint32_t>(*max_n, static_cast<uint32_t>(n));
    }
    return CKV_OK;
}

}  // namespace

extern "C" {

ckv_status ckv_pipe_store_bf16(ckv_pipe* p, const void* const* pages, const float* eps,
                               size_t count, size_t n, uint8_t* host, size_t capacity,
                               size_t* offsets, size_t* sizes, float* bounds, size_t* total,
                               uint64_t after, uint64_t* ticket, void* stream_ptr) {
    if (!p) return CKV_ERR_ARGUMENT;
    ckv_ctx* ctx = p->ctx;
    ctx->err.clear();
    if (!pages || !host || !offsets || !sizes || !bounds || !total || !fits_u32(n) || n == 0)
        return fail(ctx, CKV_ERR_ARGUMENT, "invalid pipeline store arguments");
    if (ckv_status s = check_fixed(ctx, "pipeline store")) return s;
    DeviceGuard guard(ctx->device);
    auto add = [&](Batch& b, size_t i, size_t, uint8_t* stream, size_t cap) -> ckv_status {
        const void* page = pages[i];
        if (!page || (reinterpret_cast<uintptr_t>(page) & 1u))
            return fail(ctx, CKV_ERR_ARGUMENT, "invalid page %zu", i);
        Unit u{};
        u.elems = page;
        u.stream = stream;
        u.capacity = cap;
        u.n = static_cast<uint32_t>(n);
        u.eb = eps_of(ctx, eps, i);
        b.units.push_back(u);
        return CKV_OK;
    };
    return pipe_store_units(p, count, 1, {identity_map()}, static_cast<uint32_t>(n), host,
                            capacity, offsets, sizes, bounds, total, after, ticket,
                            static_cast<cudaStream_t>(stream_ptr), add);
}

ckv_status ckv_pipe_restore_bf16(ckv_pipe* p, const uint8_t* host, const size_t* offsets,
                                 const size_t* sizes, const float* bounds, size_t count, size_t n,
                                 void* const* dst, uint64_t after, uint64_t* ticket,
                                 void* stream_ptr) {
    if (!p) return CKV_ERR_ARGUMENT;
    ckv_ctx* ctx = p->ctx;
    ctx->err.clear();
    if (!host || !offsets || !sizes || !bounds || !dst || !fits_u32(n) || n == 0)
        return fail(ctx, CKV_ERR_ARGUMENT, "invalid pipeline restore arguments");
    if (ckv_status s = check_fixed(ctx, "pipeline restore")) return s;
    DeviceGuard guard(ctx->device);
    for (size_t i = 0; i < count; ++i)
        if (!dst[i] || (reinterpret_cast<uintptr_t>(dst[i]) & 1u))
            return fail(ctx, CKV_ERR_ARGUMENT, "invalid restored page %zu", i);
    auto add = [&](Batch& b, size_t i, size_t, uint8_t* stream, size_t size) -> ckv_status {
        Unit u{};
        u.elems = dst[i];
        u.stream = stream;
        u.capacity = size;
        u.n = static_cast<uint32_t>(n);
        u.eb = bounds[i];
        b.units.push_back(u);
        return CKV_OK;
    };
    return pipe_restore_units(p, host, offsets, sizes, count, 1, {identity_map()},
                              static_cast<uint32_t>(n), after, ticket,
                              static_cast<cudaStream_t>(stream_ptr), add);
}

ckv_status ckv_pipe_store_bf16_groups(ckv_pipe* p, const void* const* pages, size_t count,
                                      const int64_t* const* layer_indices, const size_t* selected,
                                      size_t groups, size_t prefix_count, size_t source_layers,
                                      size_t elements_per_layer, const float* eps, uint8_t* host,
                                      size_t capacity, size_t* offsets, size_t* sizes,
                                      float* bounds, size_t* total, uint64_t after,
                                      uint64_t* ticket, void* stream_ptr) {
    if (!p) return CKV_ERR_ARGUMENT;
    ckv_ctx* ctx = p->ctx;
    ctx->err.clear();
    if (!pages || !host || !offsets || !sizes || !bounds || !total)
        return fail(ctx, CKV_ERR_ARGUMENT, "invalid grouped store arguments");
    if (ckv_status s = check_fixed(ctx, "grouped store")) return s;
    std::vector<Map> maps;
    uint32_t max_n = 0;
    if (ckv_status s = check_groups(ctx, layer_indices, selected, groups, prefix_count,
                                    source_layers, elements_per_layer, maps, &max_n))
        return s;
    DeviceGuard guard(ctx->device);
    auto add = [&](Batch& b, size_t i, size_t g, uint8_t* stream, size_t cap) -> ckv_status {
        const void* page = pages[i];
        if (!page || (reinterpret_cast<uintptr_t>(page) & 1u))
            return fail(ctx, CKV_ERR_ARGUMENT, "invalid page %zu", i);
        Unit u{};
        u.elems = page;
        u.stream = stream;
        u.capacity = cap;
        u.n = static_cast<uint32_t>(prefix_count * selected[g] * elements_per_layer);
        u.map = static_cast<uint32_t>(g);
        u.eb = eps_of(ctx, eps, g);
        b.units.push_back(u);
        return CKV_OK;
    };
    return pipe_store_units(p, count, groups, maps, max_n, host, capacity, offsets, sizes, bounds,
                            total, after, ticket, static_cast<cudaStream_t>(stream_ptr), add);
}

ckv_status ckv_pipe_restore_bf16_groups(ckv_pipe* p, const uint8_t* host, const size_t* offsets,
                                        const size_t* sizes, const float* bounds, size_t count,
                                        const int64_t* const* layer_indices,
                                        const size_t* selected, size_t groups,
                                        size_t prefix_count, size_t source_layers,
                                        size_t elements_per_layer, void* const* pages,
                                        uint64_t after, uint64_t* ticket, void* stream_ptr) {
    if (!p) return CKV_ERR_ARGUMENT;
    ckv_ctx* ctx = p->ctx;
    ctx->err.clear();
    if (!host || !offsets || !sizes || !bounds || !pages)
        return fail(ctx, CKV_ERR_ARGUMENT, "invalid grouped restore arguments");
    if (ckv_status s = check_fixed(ctx, "grouped restore")) return s;
    std::vector<Map> maps;
    uint32_t max_n = 0;
    if (ckv_status s = check_groups(ctx, layer_indices, selected, groups, prefix_count,
                                    source_layers, elements_per_layer, maps, &max_n))
        return s;
    DeviceGuard guard(ctx->device);
    for (size_t i = 0; i < count; ++i)
        if (!pages[i] || (reinterpret_cast<uintptr_t>(pages[i]) & 1u))
            return fail(ctx, CKV_ERR_ARGUMENT, "invalid restored page %zu", i);
    auto add = [&](Batch& b, size_t i, size_t g, uint8_t* stream, size_t size) -> ckv_status {
        Unit u{};
        u.elems = pages[i];
        u.stream = stream;
        u.capacity = size;
        u.n = static_cast<uint32_t>(prefix_count * selected[g] * elements_per_layer);
        u.map = static_cast<uint32_t>(g);
        u.eb = bounds[i * groups + g];
        b.units.push_back(u);
        return CKV_OK;
    };
    return pipe_restore_units(p, host, offsets, sizes, count, groups, maps, max_n, after, ticket,
                              static_cast<cudaStream_t>(stream_ptr), add);
}

size_t ckv_pipe_host_capacity_groups(size_t count, const size_t* selected, size_t groups,
                                     size_t prefix_count, size_t elements_per_layer) {
    size_t per_page = 0;
    for (size_t g = 0; g < groups; ++g)
        per_page += worst_page(prefix_count * selected[g] * elements_per_layer) + 16;
    return count * per_page;
}

}  // extern "C"

namespace {

// Store whose per-chunk device step needs no host synchronisation (every
// page has the same stored size `stride`, a multiple of 16): stage(k, c0,
// cnt, dst) enqueues on p->s_enc the writing of pages c0..c0+cnt-1 into dst,
// one every `stride` bytes.  Chunks are copied out as they are staged.
template <typename Stage>
ckv_status pipe_store_fixed(ckv_pipe* p, size_t count, size_t stride, uint8_t* host,
                            size_t capacity, size_t* offsets, size_t* total, uint64_t after,
                            uint64_t* ticket, cudaStream_t caller, Stage stage) {
    ckv_ctx* ctx = p->ctx;
    *total = 0;
    if (count == 0) return pipe_issue(p, caller, ticket);
    if (count * stride > capacity)
        return fail(ctx, CKV_ERR_CAPACITY, "host buffer of %zu bytes too small (%zu needed)", capacity,
                    count * stride);
    if (ckv_status st = pipe_staging(p, stride)) return st;
    cudaError_t e = cudaEventRecord(p->ev_in, caller);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(p->s_enc, p->ev_in, 0);
    if (e != cudaSuccess) return cuda_fail(ctx, "ordering the pipeline store", e);
    if (ckv_status st = pipe_after(p, after, p->s_d2h)) return st;
    size_t pos = 0;
    for (size_t c0 = 0; c0 < count; c0 += p->chunk) {
        const int k = static_cast<int>(p->store_seq++ & 1u);
        const size_t cnt = std::min(p->chunk, count - c0);
        if (p->copied_used[k] && (e = cudaStreamWaitEvent(p->s_enc, p->ev_copied[k], 0)))
            return cuda_fail(ctx, "ordering the pipeline store", e);
        if (ckv_status st = stage(k, c0, cnt, p->packed[k])) return st;
        e = cudaEventRecord(p->ev_packed[k], p->s_enc);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(p->s_d2h, p->ev_packed[k], 0);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(host + pos, p->packed[k], cnt * stride, cudaMemcpyDeviceToHost,
                                p->s_d2h);
        if (e == cudaSuccess) e = cudaEventRecord(p->ev_copied[k], p->s_d2h);
        if (e != cudaSuccess) return cuda_fail(ctx, "pipeline store copy", e);
        p->copied_used[k] = true;
        for (size_t i = 0; i < cnt; ++i) offsets[c0 + i] = pos + i * stride;
        pos += cnt * stride;
    }
    *total = pos;
    return pipe_issue(p, p->s_d2h, ticket);
}

// Restore of pages stored `bytes` each at offsets[] of the host buffer:
// each chunk's span is copied into a landing buffer, then unstage(k, c0, cnt,
// land, lo) enqueues on p->s_dec the writing of its pages (page i's bytes sit
// at land + offsets[i] - lo).
template <typename Unstage>
ckv_status pipe_restore_fixed(ckv_pipe* p, const uint8_t* host, const size_t* offsets,
                              size_t count, size_t bytes, void* const* dst, uint64_t after,
                              uint64_t* ticket, cudaStream_t caller, Unstage unstage) {
    ckv_ctx* ctx = p->ctx;
    if (count == 0) return pipe_issue(p, caller, ticket);
    size_t span_max = 0;
    for (size_t c0 = 0; c0 < count; c0 += p->chunk) {
        const size_t cnt = std::min(p->chunk, count - c0);
        size_t lo = SIZE_MAX, hi = 0;
        for (size_t i = c0; i < c0 + cnt; ++i) {
            if ((offsets[i] & 3u) || !dst[i] || (reinterpret_cast<uintptr_t>(dst[i]) & 1u))
                return fail(ctx, CKV_ERR_ARGUMENT, "invalid restored page %zu", i);
            lo = std::min(lo, offsets[i]);
            hi = std::max(hi, offsets[i] + bytes);
        }
        span_max = std::max(span_max, hi - (lo & ~size_t(15)));
    }
    if (ckv_status st = pipe_landing(p, span_max)) return st;
    cudaError_t e = cudaEventRecord(p->ev_in, caller);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(p->s_dec, p->ev_in, 0);
    if (e != cudaSuccess) return cuda_fail(ctx, "ordering the pipeline restore", e);
    if (ckv_status st = pipe_after(p, after, p->s_h2d)) return st;
    for (size_t c0 = 0; c0 < count; c0 += p->chunk) {
        const int k = static_cast<int>(p->restore_seq++ & 1u);
        const size_t cnt = std::min(p->chunk, count - c0);
        size_t lo = SIZE_MAX, hi = 0;
        for (size_t i = c0; i < c0 + cnt; ++i) {
            lo = std::min(lo, offsets[i]);
            hi = std::max(hi, offsets[i] + bytes);
        }
        lo &= ~size_t(15);
        if (p->decoded_used[k] && (e = cudaStreamWaitEvent(p->s_h2d, p->ev_decoded[k], 0)))
            return cuda_fail(ctx, "ordering the pipeline restore", e);
        e = cudaMemcpyAsync(p->land[k], host + lo, hi - lo, cudaMemcpyHostToDevice, p->s_h2d);
        if (e == cudaSuccess) e = cudaEventRecord(p->ev_landed[k], p->s_h2d);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(p->s_dec, p->ev_landed[k], 0);
        if (e != cudaSuccess) return cuda_fail(ctx, "pipeline restore copy", e);
        if (ckv_status st = unstage(k, c0, cnt, p->land[k], lo)) return st;
        if ((e = cudaEventRecord(p->ev_decoded[k], p->s_dec)))
            return cuda_fail(ctx, "pipeline restore", e);
        p->decoded_used[k] = true;
    }
    uint64_t t = 0;
    if (ckv_status st = pipe_issue(p, p->s_dec, &t)) return st;
    e = cudaStreamWaitEvent(caller, pipe_ticket_event(p, t), 0);
    if (e != cudaSuccess) return cuda_fail(ctx, "joining the pipeline restore", e);
    if (ticket) *ticket = t;
    return CKV_OK;
}

// Descriptors of one launch in the next staging slot, copied to the device
// on `stream` by the fetch kernel; `extra` zeroed bytes follow them.
template <typename D>
ckv_status stage_descriptors(ckv_ctx* ctx, size_t count, size_t extra, cudaStream_t stream,
                             Slot** slot, D** host, D** dev, uint8_t** extra_dev) {
    const size_t body = align16(count * sizeof(D));
    const size_t need = body + align16(extra);
    if (ckv_status st = acquire_slot(ctx, need, slot)) return st;
    *host = reinterpret_cast<D*>((*slot)->host);
    *dev = reinterpret_cast<D*>((*slot)->dev);
    if (extra_dev) *extra_dev = (*slot)->dev + body;
    memset((*slot)->host + body, 0, align16(extra));
    (void)stream;
    return CKV_OK;
}

ckv_status fetch_descriptors(ckv_ctx* ctx, Slot* slot, size_t bytes, cudaStream_t stream) {
    cudaError_t e = ckv::launch_fetch(slot->host_dev, slot->dev, align16(bytes), stream);
    if (e != cudaSuccess) return cuda_fail(ctx, "uploading descriptors", e);
    return CKV_OK;
}

size_t int8_stride(size_t n) { return align16(ckv::align4(static_cast<uint32_t>(n)) + 4); }

}  // namespace

extern "C" {

ckv_status ckv_pipe_store_int8(ckv_pipe* p, const void* const* pages, size_t count, size_t n,
                               uint8_t* host, size_t capacity, size_t* offsets, size_t* sizes,
                               size_t* total, uint64_t after, uint64_t* ticket, void* stream_ptr) {
    if (!p) return CKV_ERR_ARGUMENT;
    ckv_ctx* ctx = p->ctx;
    ctx->err.clear();
    if (!pages || !host || !offsets || !sizes || !total || !fits_u32(n) || n == 0 ||
        n > 0xfffffff0u)
        return fail(ctx, CKV_ERR_ARGUMENT, "invalid INT8 store arguments");
    DeviceGuard guard(ctx->device);
    const size_t stride = int8_stride(n);
    const uint32_t n32 = static_cast<uint32_t>(n);
    auto stage = [&](int, size_t c0, size_t cnt, uint8_t* dst) -> ckv_status {
        Slot* slot = nullptr;
        ckv::Int8Unit *units = nullptr, *dunits = nullptr;
        uint8_t* amax = nullptr;
        if (ckv_status st = stage_descriptors(ctx, cnt, cnt * 4, p->s_enc, &slot, &units, &dunits, &amax))
            return st;
        for (size_t i = 0; i < cnt; ++i) {
            const void* page = pages[c0 + i];
            if (!page || (reinterpret_cast<uintptr_t>(page) & 1u))
                return fail(ctx, CKV_ERR_ARGUMENT, "invalid page %zu", c0 + i);
            units[i] = ckv::Int8Unit{page, dst + i * stride,
                                     reinterpret_cast<uint32_t*>(amax) + i, n32, 0u};
        }
        if (ckv_status st = fetch_descriptors(ctx, slot, align16(cnt * sizeof(ckv::Int8Unit)) + align16(cnt * 4), p->s_enc))
            return st;
        timing_begin(ctx, 3, p->s_enc);
        cudaError_t e = ckv::launch_int8_encode(dunits, static_cast<uint32_t>(cnt), n32, p->s_enc);
        timing_end(ctx, 3, p->s_enc);
        release(slot, p->s_enc);
        if (e != cudaSuccess) return cuda_fail(ctx, "INT8 encode launch", e);
        return CKV_OK;
    };
    ckv_status st = pipe_store_fixed(p, count, stride, host, capacity, offsets, total, after, ticket,
                                     static_cast<cudaStream_t>(stream_ptr), stage);
    if (st == CKV_OK)
        for (size_t i = 0; i < count; ++i) sizes[i] = ckv::align4(n32) + 4;
    return st;
}

ckv_status ckv_pipe_restore_int8(ckv_pipe* p, const uint8_t* host, const size_t* offsets,
                                 size_t count, size_t n, void* const* dst, uint64_t after,
                                 uint64_t* ticket, void* stream_ptr) {
    if (!p) return CKV_ERR_ARGUMENT;
    ckv_ctx* ctx = p->ctx;
    ctx->err.clear();
    if (!host || !offsets || !dst || !fits_u32(n) || n == 0 || n > 0xfffffff0u)
        return fail(ctx, CKV_ERR_ARGUMENT, "invalid INT8 restore arguments");
    DeviceGuard guard(ctx->device);
    const uint32_t n32 = static_cast<uint32_t>(n);
    auto unstage = [&](int, size_t c0, size_t cnt, uint8_t* land, size_t lo) -> ckv_status {
        Slot* slot = nullptr;
        ckv::Int8Unit *units = nullptr, *dunits = nullptr;
        if (ckv_status st = stage_descriptors<ckv::Int8Unit>(ctx, cnt, 0, p->s_dec, &slot, &units,
                                                             &dunits, nullptr))
            return st;
        for (size_t i = 0; i < cnt; ++i)
            units[i] = ckv::Int8Unit{dst[c0 + i], land + (offsets[c0 + i] - lo), nullptr, n32, 0u};
        if (ckv_status st = fetch_descriptors(ctx, slot, cnt * sizeof(ckv::Int8Unit), p->s_dec))
            return st;
        timing_begin(ctx, 4, p->s_dec);
        cudaError_t e = ckv::launch_int8_decode(dunits, static_cast<uint32_t>(cnt), n32, p->s_dec);
        timing_end(ctx, 4, p->s_dec);
        release(slot, p->s_dec);
        if (e != cudaSuccess) return cuda_fail(ctx, "INT8 decode launch", e);
        return CKV_OK;
    };
    return pipe_restore_fixed(p, host, offsets, count, ckv::align4(n32) + 4, dst, after, ticket,
                              static_cast<cudaStream_t>(stream_ptr), unstage);
}

ckv_status ckv_pipe_store_raw(ckv_pipe* p, const void* const* pages, size_t count,
                              size_t page_bytes, uint8_t* host, size_t capacity, size_t* offsets,
                              size_t* total, uint64_t after, uint64_t* ticket, void* stream_ptr) {
    if (!p) return CKV_ERR_ARGUMENT;
    ckv_ctx* ctx = p->ctx;
    ctx->err.clear();
    if (!pages || !host || !offsets || !total || page_bytes == 0)
        return fail(ctx, CKV_ERR_ARGUMENT, "invalid raw store arguments");
    DeviceGuard guard(ctx->device);
    const size_t stride = align16(page_bytes);
    auto stage = [&](int, size_t c0, size_t cnt, uint8_t* dst) -> ckv_status {
        Slot* slot = nullptr;
        ckv::CopyUnit *units = nullptr, *dunits = nullptr;
        if (ckv_status st = stage_descriptors<ckv::CopyUnit>(ctx, cnt, 0, p->s_enc, &slot, &units,
                                                             &dunits, nullptr))
            return st;
        for (size_t i = 0; i < cnt; ++i) {
            if (!pages[c0 + i]) return fail(ctx, CKV_ERR_ARGUMENT, "null page %zu", c0 + i);
            units[i] = ckv::CopyUnit{static_cast<const uint8_t*>(pages[c0 + i]), dst + i * stride,
                                     page_bytes};
        }
        if (ckv_status st = fetch_descriptors(ctx, slot, cnt * sizeof(ckv::CopyUnit), p->s_enc))
            return st;
        timing_begin(ctx, 5, p->s_enc);
        cudaError_t e = ckv::launch_copy(dunits, static_cast<uint32_t>(cnt), page_bytes, p->s_enc);
        timing_end(ctx, 5, p->s_enc);
        release(slot, p->s_enc);
        if (e != cudaSuccess) return cuda_fail(ctx, "raw gather launch", e);
        return CKV_OK;
    };
    return pipe_store_fixed(p, count, stride, host, capacity, offsets, total, after, ticket,
                            static_cast<cudaStream_t>(stream_ptr), stage);
}

ckv_status ckv_pipe_restore_raw(ckv_pipe* p, const uint8_t* host, const size_t* offsets,
                                size_t count, size_t page_bytes, void* const* dst, uint64_t after,
                                uint64_t* ticket, void* stream_ptr) {
    if (!p) return CKV_ERR_ARGUMENT;
    ckv_ctx* ctx = p->ctx;
    ctx->err.clear();
    if (!host || !offsets || !dst || page_bytes == 0)
        return fail(ctx, CKV_ERR_ARGUMENT, "invalid raw restore arguments");
    DeviceGuard guard(ctx->device);
    auto unstage = [&](int, size_t c0, size_t cnt, uint8_t* land, size_t lo) -> ckv_status {
        Slot* slot = nullptr;
        ckv::CopyUnit *units = nullptr, *dunits = nullptr;
        if (ckv_status st = stage_descriptors<ckv::CopyUnit>(ctx, cnt, 0, p->s_dec, &slot, &units,
                                                             &dunits, nullptr))
            return st;
        for (size_t i = 0; i < cnt; ++i)
            units[i] = ckv::CopyUnit{land + (offsets[c0 + i] - lo),
                                     static_cast<uint8_t*>(dst[c0 + i]), page_bytes};
        if (ckv_status st = fetch_descriptors(ctx, slot, cnt * sizeof(ckv::CopyUnit), p->s_dec))
            return st;
        timing_begin(ctx, 5, p->s_dec);
        cudaError_t e = ckv::launch_copy(dunits, static_cast<uint32_t>(cnt), page_bytes, p->s_dec);
        timing_end(ctx, 5, p->s_dec);
        release(slot, p->s_dec);
        if (e != cudaSuccess) return cuda_fail(ctx, "raw scatter launch", e);
        return CKV_OK;
    };
    return pipe_restore_fixed(p, host, offsets, count, page_bytes, dst, after, ticket,
                              static_cast<cudaStream_t>(stream_ptr), unstage);
}

size_t ckv_pipe_host_capacity_int8(size_t count, size_t n) { return count * int8_stride(n); }

size_t ckv_pipe_host_capacity_raw(size_t count, size_t page_bytes) {
    return count * align16(page_bytes);
}

ckv_status ckv_pipe_join(ckv_pipe* p, uint64_t ticket, void* stream) {
    if (!p) return CKV_ERR_ARGUMENT;
    DeviceGuard guard(p->ctx->device);
    return pipe_after(p, ticket, static_cast<cudaStream_t>(stream));
}

ckv_status ckv_pipe_record(ckv_pipe* p, void* stream, uint64_t* ticket) {
    if (!p || !ticket) return CKV_ERR_ARGUMENT;
    DeviceGuard guard(p->ctx->device);
    return pipe_issue(p, static_cast<cudaStream_t>(stream), ticket);
}

ckv_status ckv_pipe_wait(ckv_pipe* p, uint64_t ticket) {
    if (!p) return CKV_ERR_ARGUMENT;
    if (!ticket) return CKV_OK;
    if (ticket >= p->next_ticket) return fail(p->ctx, CKV_ERR_ARGUMENT, "unknown ticket");
    if (pipe_retired(p, ticket)) return CKV_OK;
    DeviceGuard guard(p->ctx->device);
    cudaError_t e = cudaEventSynchronize(pipe_ticket_event(p, ticket));
    if (e != cudaSuccess) return cuda_fail(p->ctx, "waiting for a pipeline ticket", e);
    return CKV_OK;
}

int ckv_pipe_done(ckv_pipe* p, uint64_t ticket) {
    if (!p || ticket >= p->next_ticket) return -1;
    if (!ticket || pipe_retired(p, ticket)) return 1;
    DeviceGuard guard(p->ctx->device);
    const cudaError_t e = cudaEventQuery(pipe_ticket_event(p, ticket));
    if (e == cudaSuccess) return 1;
    // the event may already be newer work's: the ticket retired meanwhile
    if (e == cudaErrorNotReady) return pipe_retired(p, ticket) ? 1 : 0;
    return -1;
}

size_t ckv_pipe_host_capacity(size_t count, size_t n) {
    return count * (worst_page(n) + 16);
}

}  // extern "C"
