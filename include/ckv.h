/*
 * ckv.h -- C ABI of libckv, the B200 (sm_100a) fixed-mode KV-page codec.
 *
 * Drop-in boundary for the reference's CuSZpWrapper
 * (integration/cuszp_wrapper/cuszp_wrapper.h:9-158, exposed to Python by
 * integration/cuszp_wrapper/pybind11_bindings.cpp:9-264).  Every wrapper
 * method has one entry point here with the same arguments, as plain
 * pointers and sizes: tensors become device pointers plus element counts,
 * std::vector<torch::Tensor> becomes a host array of device pointers, and
 * the Python-visible outputs (sizes, resolved bounds) are written to caller
 * host arrays.  No torch types cross the boundary.
 *
 * Conventions
 *   - Every call returns CKV_OK (0) or a nonzero ckv_status; the message is
 *     available from ckv_last_error().  The reference returns bool and
 *     prints to stderr; the Python module maps !CKV_OK to False plus the
 *     message on stderr.
 *   - `stream` is a cudaStream_t (0 = legacy default stream).  Compression
 *     calls block until sizes and bounds are on the host, as the reference
 *     does (cuszp_wrapper.cpp:530); decompression calls only enqueue work.
 *   - Caller owns all data buffers.  A context owns grow-only device and
 *     pinned-host workspaces and is not thread-safe (one per thread), like
 *     one CuSZpWrapper instance.
 *   - Bitstreams are byte-identical to the reference's batched BF16 kernels
 *     (cuszp_batched_fixed.cu), except that rate bytes of blocks past the
 *     last element -- never written by the reference -- are written as 0.
 */
#ifndef CKV_H
#define CKV_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define CKV_API __attribute__((visibility("default")))
#else
#define CKV_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef int ckv_status;
#define CKV_OK 0
#define CKV_ERR_ARGUMENT 1      /* invalid argument / precondition */
#define CKV_ERR_UNSUPPORTED 2   /* configuration outside the fixed 1D path */
#define CKV_ERR_CUDA 3          /* CUDA runtime error */
#define CKV_ERR_CAPACITY 4      /* compressed data larger than its buffer */
#define CKV_ERR_STREAM 5        /* corrupt or truncated bitstream */
#define CKV_ERR_INTERNAL 6      /* device-side consistency check failed */

/* cuszp_dim_t / cuszp_mode_t / cuszp_type_t (pybind11_bindings.cpp:13-28).
 * Upstream cuSZp's header is not vendored by the reference, so its numeric
 * values cannot be read there; these follow the order in which the
 * reference binds them (FIXED, PLAIN, OUTLIER: pybind11_bindings.cpp:19-22;
 * DIM_1D..3D: :13-17; FLOAT, DOUBLE: :24-27).  oracle/ref_shim/cuSZp.h,
 * which stands in for that header when the reference's kernels are built as
 * a test oracle, uses the same values. */
#define CKV_DIM_1D 0
#define CKV_DIM_2D 1
#define CKV_DIM_3D 2
#define CKV_MODE_FIXED 0
#define CKV_MODE_PLAIN 1
#define CKV_MODE_OUTLIER 2
#define CKV_TYPE_FLOAT 0
#define CKV_TYPE_DOUBLE 1

/* CuSZpWrapper::CompressionConfig (cuszp_wrapper.h:11-17). */
typedef struct {
    float error_bound;          /* default 1e-4 */
    int use_relative_error;     /* default 1 */
    int processing_dim;         /* CKV_DIM_* */
    int encoding_mode;          /* CKV_MODE_*; only FIXED is implemented */
    int data_type;              /* CKV_TYPE_*; only FLOAT is implemented */
} ckv_config;

typedef struct ckv_ctx ckv_ctx;

/* CuSZpWrapper(config, device_id)   cuszp_wrapper.cpp:23-39 */
CKV_API ckv_status ckv_create(const ckv_config* config, int device_id, ckv_ctx** out);
/* ~CuSZpWrapper()                   cuszp_wrapper.cpp:41-66 */
CKV_API void ckv_destroy(ckv_ctx* ctx);
/* get_config / update_config        cuszp_wrapper.h:126-127 */
CKV_API ckv_status ckv_get_config(const ckv_ctx* ctx, ckv_config* out);
CKV_API ckv_status ckv_update_config(ckv_ctx* ctx, const ckv_config* config);
/* Message of the last failed call on this context ("" if none). */
CKV_API const char* ckv_last_error(const ckv_ctx* ctx);
/* estimate_compressed_buffer_size   cuszp_wrapper.cpp:1319-1321 (2 * bytes) */
CKV_API size_t ckv_estimate_compressed_buffer_size(size_t original_bytes);
/* Upper bound of the compressed size of n elements (every block at rate 31). */
CKV_API size_t ckv_max_compressed_size(size_t n);

/* compress(input, buffer, eps_override)   cuszp_wrapper.cpp:216-325.
 * FP32 input of n elements, fixed mode.  The reference reallocates a
 * too-small buffer; here the caller provides `capacity` bytes and gets
 * CKV_ERR_CAPACITY (with *size = needed bytes) if it is too small. */
CKV_API ckv_status ckv_compress(ckv_ctx* ctx, const float* input, size_t n,
                        uint8_t* out, size_t capacity, float eps_override,
                        size_t* size, float* bound, void* stream);

/* compress_batch_fixed(inputs, outputs, eps)   cuszp_wrapper.cpp:327-429.
 * `eps` may be NULL (config bound); eps[i] <= 0 also means config bound. */
CKV_API ckv_status ckv_compress_batch_fixed(ckv_ctx* ctx, const float* const* inputs,
                                    uint8_t* const* outputs, const float* eps,
                                    size_t batch, size_t n, size_t capacity,
                                    size_t* sizes, float* bounds, void* stream);

/* compress_batch_fixed_bf16(inputs, outputs, eps)  cuszp_wrapper.cpp:431-544 */
CKV_API ckv_status ckv_compress_batch_fixed_bf16(ckv_ctx* ctx, const void* const* inputs,
                                         uint8_t* const* outputs, const float* eps,
                                         size_t batch, size_t n, size_t capacity,
                                         size_t* sizes, float* bounds, void* stream);

/* compress_batch_fixed_bf16_indexed(...)       cuszp_wrapper.cpp:548-681.
 * Pages are [prefix_count][source_layers][elements_per_layer] BF16; unit i
 * is layers layer_indices[0..selected) (device int64 array) of page i.
 * Every index must lie in [0, source_layers): the values live on the device
 * and, as in the reference (cuszp_batched_fixed.cu:33-50), are not checked
 * (this applies to every call below that takes layer indices). */
CKV_API ckv_status ckv_compress_batch_fixed_bf16_indexed(
    ckv_ctx* ctx, const void* const* inputs, uint8_t* const* outputs,
    const int64_t* layer_indices, size_t selected, size_t prefix_count,
    size_t source_layers, size_t elements_per_layer, const float* eps,
    size_t batch, size_t capacity, size_t* sizes, float* bounds, void* stream);

/* compress_batch_fixed_bf16_indexed_groups(...) cuszp_wrapper.cpp:683-868.
 * Group g covers group_sizes[g] consecutive units and selects
 * selected[g] layers from layer_indices[g] (device int64 arrays).  All
 * groups go into ONE launch here (the reference launches per group).
 * capacities[i] is unit i's buffer size in bytes. */
CKV_API ckv_status ckv_compress_batch_fixed_bf16_indexed_groups(
    ckv_ctx* ctx, const void* const* inputs, uint8_t* const* outputs,
    const int64_t* const* layer_indices, const size_t* selected,
    const size_t* group_sizes, size_t groups, size_t prefix_count,
    size_t source_layers, size_t elements_per_layer, const float* eps,
    size_t batch, const size_t* capacities, size_t* sizes, float* bounds,
    void* stream);

/* decompress(buffer, size, output, bound)      cuszp_wrapper.cpp:870-943.
 * FP32 output of n elements, fixed mode. */
CKV_API ckv_status ckv_decompress(ckv_ctx* ctx, const uint8_t* in, size_t size,
                          float* out, size_t n, float bound, void* stream);

/* decompress_batch(buffers, sizes, outputs, bounds) cuszp_wrapper.cpp:944-1033.
 * FP32 outputs, n[i] elements each; one launch for the whole batch. */
CKV_API ckv_status ckv_decompress_batch(ckv_ctx* ctx, const uint8_t* const* ins,
                                const size_t* sizes, float* const* outs,
                                const size_t* n, const float* bounds,
                                size_t batch, void* stream);

/* decompress_batch_fixed_bf16(...)             cuszp_wrapper.cpp:1034-1110.
 * Page i decodes to out + i * n (BF16); out holds out_numel elements. */
CKV_API ckv_status ckv_decompress_batch_fixed_bf16(ckv_ctx* ctx, const uint8_t* const* ins,
                                           const size_t* sizes, size_t batch,
                                           void* out, size_t out_numel, size_t n,
                                           const float* bounds, void* stream);

/* decompress_batch_fixed_bf16_scatter(...)     cuszp_wrapper.cpp:1111-1212.
 * Page i decodes into outs[i * per_page + d], elements_per_dest each. */
CKV_API ckv_status ckv_decompress_batch_fixed_bf16_scatter(
    ckv_ctx* ctx, const uint8_t* const* ins, const size_t* sizes, size_t batch,
    void* const* outs, size_t out_count, size_t n, size_t per_page,
    size_t elements_per_dest, const float* bounds, void* stream);

/* decompress_batch_fixed_bf16_indexed_scatter(...) cuszp_wrapper.cpp:1214-1313.
 * Unit i decodes into layers layer_indices[0..selected) of page outs[i]. */
CKV_API ckv_status ckv_decompress_batch_fixed_bf16_indexed_scatter(
    ckv_ctx* ctx, const uint8_t* const* ins, const size_t* sizes, size_t batch,
    void* const* outs, const int64_t* layer_indices, size_t selected,
    size_t prefix_count, size_t source_layers, size_t elements_per_layer,
    const float* bounds, void* stream);

/* ---- extensions (no counterpart in the reference wrapper) ---------------- */

/* Decode rate-0 blocks as zeros instead of leaving the destination as it was
 * (the reference decoder does not write those blocks). */
CKV_API ckv_status ckv_set_zero_fill(ckv_ctx* ctx, int zero_fill);

/* OR of the device status bits recorded by asynchronous decode calls since
 * the last call with reset != 0 (CKV_DEV_* below); waits for the work queued
 * on `stream` first. */
#define CKV_DEV_CAPACITY 1u
#define CKV_DEV_RATE_CHECK 2u
#define CKV_DEV_BAD_STREAM 4u
#define CKV_DEV_TIMEOUT 8u
CKV_API ckv_status ckv_device_status(ckv_ctx* ctx, void* stream, int reset, uint32_t* bits);

/* Status words (CKV_DEV_* bits, 0 = fine) of each of the first `count`
 * units of the last compress call on this context, e.g. which unit did not
 * fit its buffer. */
CKV_API ckv_status ckv_unit_status(ckv_ctx* ctx, size_t count, uint32_t* out);

/* Failure-path test hook.  The next encode launch on this context withholds
 * the bound exchange of batch unit `unit` inside its thread-block cluster
 * (the cluster's first CTA sends nothing for it), so every CTA of that
 * cluster waits for data that never comes, and that cluster's waits give up
 * after `wait_polls` polls instead of the default.  Every role of that
 * cluster then stops once the copies it issued have landed and its units
 * are marked CKV_DEV_TIMEOUT; the call fails with CKV_ERR_CUDA ("a bounded
 * wait in the kernel ran out"), the other clusters' units complete
 * normally, nothing faults or hangs, and the context stays usable. */
CKV_API ckv_status ckv_test_withhold_exchange(ckv_ctx* ctx, uint32_t unit, uint32_t wait_polls);

/* Which BF16 encoder this context's compress calls use (no counterpart in
 * the reference, whose wrapper has one kernel).  Both write the same bytes,
 * sizes and bounds.  CKV_ENCODER_AUTO (the default) takes the streaming
 * encoder for batches of whole pages (every unit a contiguous, 16-byte
 * aligned page) of at most 16384 elements each, where it is faster, and the
 * clustered encoder otherwise (a large batch of whole pages may hand the
 * clustered encoder's last, nearly empty round of units, and for long
 * batches whole further rounds, to the streaming encoder, which then runs
 * beside it on the SMs no cluster holds);
 * CKV_ENCODER_CLUSTER always the clustered one alone;
 * CKV_ENCODER_STREAM the streaming one whenever the batch is whole pages.
 * The streaming encoder handles one unit per CTA and reads it twice (bound,
 * then bit planes); the clustered one spreads a unit over a thread-block
 * cluster and reads it once.  When a unit does not fit its buffer both fail
 * with CKV_ERR_CAPACITY and write nothing past the buffer; the clustered
 * encoder writes nothing of that unit, the streaming one may have written
 * its leading chunks. */
enum { CKV_ENCODER_AUTO = 0, CKV_ENCODER_CLUSTER = 1, CKV_ENCODER_STREAM = 2 };
CKV_API ckv_status ckv_set_encoder(ckv_ctx* ctx, int choice);

/* Gather `count` compressed units (device pointers srcs[i], sizes[i] bytes)
 * into the device slab `dst` (capacity bytes), unit i starting at
 * offsets[i] = previous end rounded up to `align` bytes (a power of two,
 * >= 4).  Writes the offsets to the host array and the slab's used length
 * to *total.  One launch; asynchronous on `stream`.  The reference does
 * this with torch.cat (vllm_v1_compressed_offload.py:403-427). */
CKV_API ckv_status ckv_pack(ckv_ctx* ctx, const uint8_t* const* srcs, const size_t* sizes,
                            size_t count, uint8_t* dst, size_t capacity, size_t align,
                            size_t* offsets, size_t* total, void* stream);

/* Record CUDA events immediately around every kernel this context launches
 * (on the launch stream).  ckv_kernel_time returns the device duration of
 * the last launch of the given kind (0 encode, 1 decode, 2 pack, 3 INT8
 * encode, 4 INT8 decode, 5 raw page copy), in milliseconds, waiting for it to
 * finish. */
CKV_API ckv_status ckv_set_kernel_timing(ckv_ctx* ctx, int enable);
CKV_API ckv_status ckv_kernel_time(ckv_ctx* ctx, int kind, float* ms);

/* Store / restore pipeline (replaces the job path of the reference's
 * connector: CompressedPageStore.put_many_packed,
 * vllm_v1_compressed_offload.py:371-447, which compresses a whole job, packs
 * it with torch.cat into one pinned slab and synchronises; and
 * _decompress_bundles_batched, :1618-1711, which copies the whole slab back
 * before decoding; transfer_async, :2365-2385, orders the jobs).  A pipeline
 * owns its CUDA streams (compute, device-to-host, host-to-device, decode)
 * and double-buffered device staging, and runs a job in chunks of
 * `chunk_pages` pages: the device-to-host copy of chunk k overlaps the
 * compression of chunk k+1, the host-to-device copy of chunk k+1 the
 * decompression of chunk k, and a store and a restore in flight together use
 * both directions of the link.  Not thread-safe; one pipeline per context.
 * Only ckv_pipe_done and ckv_pipe_wait may be called from another thread
 * while a pipeline call runs (e.g. a poller of finished jobs). */
typedef struct ckv_pipe ckv_pipe;
CKV_API ckv_status ckv_pipe_create(ckv_ctx* ctx, size_t chunk_pages, ckv_pipe** out);
CKV_API void ckv_pipe_destroy(ckv_pipe* pipe);

/* Compresses `count` BF16 pages of n elements (eps as in
 * ckv_compress_batch_fixed_bf16) into page-locked host memory: page i at
 * host + offsets[i] (16-byte aligned, pages packed in order), *total bytes
 * used.  The compression waits for work already on `stream` (the pages);
 * the copies wait for ticket `after` (0: none), e.g. a restore still reading
 * the same host buffer.  Returns when sizes, bounds and offsets are on the
 * host and every copy is queued; *ticket completes with the last copy. */
CKV_API ckv_status ckv_pipe_store_bf16(ckv_pipe* pipe, const void* const* pages,
                                       const float* eps, size_t count, size_t n,
                                       uint8_t* host, size_t capacity, size_t* offsets,
                                       size_t* sizes, float* bounds, size_t* total,
                                       uint64_t after, uint64_t* ticket, void* stream);

/* Decompresses `count` pages from page-locked host memory (offsets, sizes
 * and bounds as a store returned them) into the BF16 pages dst[i] of n
 * elements.  The copies wait for ticket `after` (0: none), e.g. the store
 * that wrote the host buffer; the decode waits for work already on
 * `stream`, and `stream` waits for the decode (asynchronous, like
 * ckv_decompress_batch_fixed_bf16). */
CKV_API ckv_status ckv_pipe_restore_bf16(ckv_pipe* pipe, const uint8_t* host,
                                         const size_t* offsets, const size_t* sizes,
                                         const float* bounds, size_t count, size_t n,
                                         void* const* dst, uint64_t after, uint64_t* ticket,
                                         void* stream);

/* Make `stream` wait for a ticket (device side); wait for it on the host;
 * query it (1 done, 0 pending, -1 unknown).  A pipeline keeps the events of
 * its last 64 tickets: issuing a ticket first waits on the host for the one
 * 64 before it and marks it retired, so an older ticket is complete (done 1,
 * wait and join return at once).  A wait from another thread that races with
 * the issue retiring its ticket may also wait for the newer work. */
CKV_API ckv_status ckv_pipe_join(ckv_pipe* pipe, uint64_t ticket, void* stream);
/* A ticket for the work queued on `stream` so far (the caller's own copies
 * into or out of a host buffer, which later pipeline calls can then be
 * ordered after with `after`). */
CKV_API ckv_status ckv_pipe_record(ckv_pipe* pipe, void* stream, uint64_t* ticket);
CKV_API ckv_status ckv_pipe_wait(ckv_pipe* pipe, uint64_t ticket);
CKV_API int ckv_pipe_done(ckv_pipe* pipe, uint64_t ticket);

/* Host bytes that always hold `count` compressed pages of n elements. */
CKV_API size_t ckv_pipe_host_capacity(size_t count, size_t n);

/* Layer-grouped store and restore (the connector's per-layer bound profile:
 * _compress_adaptive_fixed_bundles_indexed, vllm_v1_compressed_offload.py:
 * 1286-1569, which compresses each page as one segment per layer group with
 * compress_batch_fixed_bf16_indexed_groups, and restores each group with
 * decompress_batch_fixed_bf16_indexed_scatter).  Each page
 * [prefix_count][source_layers][elements_per_layer] is stored as `groups`
 * segments: segment g holds layers layer_indices[g][0..selected[g]) (device
 * int64 arrays) of every prefix, compressed at eps[g] (NULL or <= 0: the
 * context's bound).  Segment g of page i is entry i * groups + g of
 * offsets / sizes / bounds.  The restore writes every group back into its
 * layers of pages[i], all groups of a chunk in one decode launch.  The host
 * buffer needs ckv_pipe_host_capacity_groups(...) bytes. */
CKV_API ckv_status ckv_pipe_store_bf16_groups(ckv_pipe* pipe, const void* const* pages,
                                              size_t count, const int64_t* const* layer_indices,
                                              const size_t* selected, size_t groups,
                                              size_t prefix_count, size_t source_layers,
                                              size_t elements_per_layer, const float* eps,
                                              uint8_t* host, size_t capacity, size_t* offsets,
                                              size_t* sizes, float* bounds, size_t* total,
                                              uint64_t after, uint64_t* ticket, void* stream);
CKV_API ckv_status ckv_pipe_restore_bf16_groups(ckv_pipe* pipe, const uint8_t* host,
                                                const size_t* offsets, const size_t* sizes,
                                                const float* bounds, size_t count,
                                                const int64_t* const* layer_indices,
                                                const size_t* selected, size_t groups,
                                                size_t prefix_count, size_t source_layers,
                                                size_t elements_per_layer, void* const* pages,
                                                uint64_t after, uint64_t* ticket, void* stream);
CKV_API size_t ckv_pipe_host_capacity_groups(size_t count, const size_t* selected, size_t groups,
                                             size_t prefix_count, size_t elements_per_layer);

/* The reference's comparison codecs through the same pipeline (its INT8
 * encoding, vllm_v1_compressed_offload.py:711-724 store and :2090-2116
 * restore, and its raw encoding, :1578-1615), so that they are timed on the
 * same streams, staging and copies as the fixed-mode codec.
 *
 * INT8: per page scale = max|x| / 127 (FP32; 1 for an all-zero page),
 * q = clamp(round_half_even(x / scale), -127, 127); restore writes
 * bf16_rn((float)q * scale).  A stored page is its n int8 values followed by
 * the FP32 scale at byte align4(n): sizes[i] = align4(n) + 4 (the
 * reference's numel + 4).  Offsets are 16-byte aligned.  Neither call
 * synchronises the host: every stored size is known in advance.  The host
 * buffer needs ckv_pipe_host_capacity_int8(count, n) bytes.
 *
 * Raw: the pages' bytes, page_bytes each, at 16-byte aligned offsets; the
 * host buffer needs ckv_pipe_host_capacity_raw(count, page_bytes) bytes.
 *
 * Ordering (after / ticket / stream) is as for ckv_pipe_store_bf16 and
 * ckv_pipe_restore_bf16. */
CKV_API ckv_status ckv_pipe_store_int8(ckv_pipe* pipe, const void* const* pages, size_t count,
                                       size_t n, uint8_t* host, size_t capacity, size_t* offsets,
                                       size_t* sizes, size_t* total, uint64_t after,
                                       uint64_t* ticket, void* stream);
CKV_API ckv_status ckv_pipe_restore_int8(ckv_pipe* pipe, const uint8_t* host,
                                         const size_t* offsets, size_t count, size_t n,
                                         void* const* pages, uint64_t after, uint64_t* ticket,
                                         void* stream);
CKV_API ckv_status ckv_pipe_store_raw(ckv_pipe* pipe, const void* const* pages, size_t count,
                                      size_t page_bytes, uint8_t* host, size_t capacity,
                                      size_t* offsets, size_t* total, uint64_t after,
                                      uint64_t* ticket, void* stream);
CKV_API ckv_status ckv_pipe_restore_raw(ckv_pipe* pipe, const uint8_t* host,
                                        const size_t* offsets, size_t count, size_t page_bytes,
                                        void* const* pages, uint64_t after, uint64_t* ticket,
                                        void* stream);
CKV_API size_t ckv_pipe_host_capacity_int8(size_t count, size_t n);
CKV_API size_t ckv_pipe_host_capacity_raw(size_t count, size_t page_bytes);

/* ckv_compress_batch_fixed_bf16 for callers that cannot allocate memory.
 * No counterpart in the reference.  Some callers cannot call cudaMalloc when
 * they compress: a serving engine that reserved all free HBM for its KV
 * cache at start-up (a later allocation fails or evicts cache), or code that
 * must not risk the device-wide synchronisation a cudaFree implies.  This
 * entry point needs no context and allocates nothing: its scratch (unit
 * descriptors, pointer tables, sizes, bounds, status) is one fixed
 * file-scope device array of CKV_NOALLOC_MAX_UNITS units (about 270 KB),
 * held by every GPU that loads the library until the process exits.
 * Larger batches are rejected with CKV_ERR_ARGUMENT and a message on stderr.
 * CUDA loads the library's kernels and its copy of the array on a device
 * lazily, at first use, and that allocates device memory; so call this once
 * per device with batch == 0 (every other argument is then ignored; the
 * device must be current) at start-up, before HBM is reserved and before
 * any stream capture.  That set-up call looks up the array's device address,
 * loads both encoder kernels (one for units of up to nine 64 KB slices per
 * CTA, one for larger units) and runs a built-in 32-element unit, held in
 * the array itself, through every launch a real call makes; later calls
 * then allocate nothing.  All
 * calls share the array: calls that overlap on the GPU race.  Otherwise as
 * ckv_compress_batch_fixed_bf16: `error_bound` and `relative` replace the
 * context's configuration, eps may be NULL, the call blocks until sizes and
 * bounds are on the host, and the bitstreams are identical. */
#define CKV_NOALLOC_MAX_UNITS 4096
CKV_API ckv_status ckv_compress_batch_fixed_bf16_noalloc(
    const void* const* inputs, uint8_t* const* outputs, const float* eps, size_t batch,
    size_t n, size_t capacity, float error_bound, int relative, size_t* sizes,
    float* bounds, void* stream);

/* Number of kernel launches libckv has issued since it was loaded. */
CKV_API uint64_t ckv_kernel_launches(void);

#ifdef __cplusplus
}
#endif

#endif /* CKV_H */
