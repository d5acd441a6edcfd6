// Host driver for the reference's own batched fixed-mode kernels.
//
// TEST INFRASTRUCTURE ONLY.  oracle/build.py compiles this file together
// with the reference's integration/cuszp_wrapper/cuszp_batched_fixed.cu
// (unchanged, read where it lies) into oracle/_ref/libref_fixed.so.  Tests
// use it to produce golden bitstreams and bench.py's reference arm times it;
// the product library never links it.
//
// Each entry point does what CuSZpWrapper does around the launchers
// (cuszp_wrapper.cpp:431-544, 548-681, 1034-1110, 1111-1212, 1214-1313):
// upload the pointer tables and bounds, zero the look-back state, launch on
// the given stream.  Differences, all in favour of deterministic tests:
//   * the compressed buffers are zeroed before compression so the rate
//     bytes the reference never writes (blocks past the last element) are
//     defined;
//   * sizes and bounds come back through one pinned copy each.
#include <cuda_runtime.h>
#include <cstdint>
#include <cstdio>
#include <vector>

bool launch_cuszp_compress_batch_fixed_bf16(
    const void* const* input_pages, unsigned char* const* compressed_pages,
    volatile unsigned int* compressed_offsets,
    volatile unsigned int* local_offsets, volatile int* flags,
    float* error_bounds, size_t num_elements, size_t batch_size,
    bool use_relative_error, cudaStream_t stream);
bool launch_cuszp_compress_batch_fixed_bf16_indexed(
    const void* const* input_pages, unsigned char* const* compressed_pages,
    volatile unsigned int* compressed_offsets,
    volatile unsigned int* local_offsets, volatile int* flags,
    float* error_bounds, const int64_t* layer_indices, size_t prefix_count,
    size_t source_layers, size_t elements_per_layer, size_t selected_layers,
    size_t batch_size, bool use_relative_error, cudaStream_t stream);
bool launch_cuszp_decompress_batch_fixed_bf16(
    void* output, const unsigned char* const* compressed_pages,
    volatile unsigned int* compressed_offsets,
    volatile unsigned int* local_offsets, volatile int* flags,
    const float* error_bounds, size_t num_elements, size_t batch_size,
    cudaStream_t stream);
bool launch_cuszp_decompress_batch_fixed_bf16_scatter(
    void* const* destination_pages, size_t destinations_per_page,
    size_t elements_per_destination,
    const unsigned char* const* compressed_pages,
    volatile unsigned int* compressed_offsets,
    volatile unsigned int* local_offsets, volatile int* flags,
    const float* error_bounds, size_t num_elements, size_t batch_size,
    cudaStream_t stream);
bool launch_cuszp_decompress_batch_fixed_bf16_indexed_scatter(
    void* const* destination_pages,
    const unsigned char* const* compressed_pages,
    volatile unsigned int* compressed_offsets,
    volatile unsigned int* local_offsets, volatile int* flags,
    const float* error_bounds, const int64_t* layer_indices,
    size_t prefix_count, size_t source_layers, size_t elements_per_layer,
    size_t selected_layers, size_t batch_size, cudaStream_t stream);

namespace {

constexpr size_t kGroup = 32 * 1024;

struct Workspace {
    unsigned int* cmp = nullptr;
    unsigned int* local = nullptr;
    int* flags = nullptr;
    void** ptrs_a = nullptr;
    void** ptrs_b = nullptr;
    float* ebs = nullptr;
    unsigned int* sizes_host = nullptr;
    float* ebs_host = nullptr;
    size_t entries = 0, ptrs = 0, count = 0;

    bool reserve(size_t e, size_t p, size_t c) {
        if (e > entries) {
            cudaFree(cmp); cudaFree(local); cudaFree(flags);
            if (cudaMalloc(&cmp, e * 4) || cudaMalloc(&local, e * 4) ||
                cudaMalloc(&flags, e * 4)) return false;
            entries = e;
        }
        if (p > ptrs) {
            cudaFree(ptrs_a); cudaFree(ptrs_b);
            if (cudaMalloc(&ptrs_a, p * sizeof(void*)) ||
                cudaMalloc(&ptrs_b, p * sizeof(void*))) return false;
            ptrs = p;
        }
        if (c > count) {
            cudaFree(ebs); cudaFreeHost(sizes_host); cudaFreeHost(ebs_host);
            if (cudaMalloc(&ebs, c * 4) || cudaMallocHost(&sizes_host, c * 4) ||
                cudaMallocHost(&ebs_host, c * 4)) return false;
            count = c;
        }
        return true;
    }
    void zero(size_t e, cudaStream_t s) {
        cudaMemsetAsync(cmp, 0, e * 4, s);
        cudaMemsetAsync(local, 0, e * 4, s);
        cudaMemsetAsync(flags, 0, e * 4, s);
    }
};

Workspace g_ws;

size_t groups_of(size_t n) { return (n + kGroup - 1) / kGroup; }

}  // namespace

extern "C" {

// Compress `batch` BF16 pages (device pointers in host array `inputs`) into
// `outputs` (device pointers, capacity `out_capacity` bytes each).
// zero_outputs != 0 clears the outputs first (golden generation); the
// reference wrapper does not, and neither does the benchmark.
// layer_indices == nullptr selects the plain kernel; otherwise the indexed
// kernel over `selected` layers.  eps[i] is the requested bound per page.
// Writes sizes and resolved bounds to host arrays.  Returns 0 on success.
int ref_compress_bf16(const void* const* inputs, unsigned char* const* outputs,
                      size_t out_capacity, size_t batch, size_t n,
                      const float* eps, int relative,
                      const int64_t* layer_indices, size_t selected,
                      size_t prefix_count, size_t source_layers,
                      size_t elements_per_layer, size_t* sizes,
                      float* bounds, void* stream_ptr, int zero_outputs) {
    cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
    size_t logical = layer_indices
        ? prefix_count * selected * elements_per_layer : n;
    size_t g = groups_of(logical);
    size_t entries = (g + 1) * batch;
    if (!g_ws.reserve(entries, batch, batch)) return 1;
    if (zero_outputs)
        for (size_t i = 0; i < batch; ++i)
            cudaMemsetAsync(outputs[i], 0, out_capacity, stream);
    cudaMemcpyAsync(g_ws.ptrs_a, inputs, batch * sizeof(void*),
                    cudaMemcpyHostToDevice, stream);
    cudaMemcpyAsync(g_ws.ptrs_b, outputs, batch * sizeof(void*),
                    cudaMemcpyHostToDevice, stream);
    cudaMemcpyAsync(g_ws.ebs, eps, batch * 4, cudaMemcpyHostToDevice, stream);
    g_ws.zero(entries, stream);
    bool ok;
    if (layer_indices) {
        ok = launch_cuszp_compress_batch_fixed_bf16_indexed(
            g_ws.ptrs_a, reinterpret_cast<unsigned char* const*>(g_ws.ptrs_b),
            g_ws.cmp, g_ws.local, g_ws.flags, g_ws.ebs, layer_indices,
            prefix_count, source_layers, elements_per_layer, selected, batch,
            relative != 0, stream);
    } else {
        ok = launch_cuszp_compress_batch_fixed_bf16(
            g_ws.ptrs_a, reinterpret_cast<unsigned char* const*>(g_ws.ptrs_b),
            g_ws.cmp, g_ws.local, g_ws.flags, g_ws.ebs, n, batch,
            relative != 0, stream);
    }
    if (!ok) return 2;
    cudaMemcpyAsync(g_ws.ebs_host, g_ws.ebs, batch * 4,
                    cudaMemcpyDeviceToHost, stream);
    for (size_t i = 0; i < batch; ++i)
        cudaMemcpyAsync(g_ws.sizes_host + i, g_ws.cmp + i * (g + 1) + g, 4,
                        cudaMemcpyDeviceToHost, stream);
    if (cudaStreamSynchronize(stream) != cudaSuccess) return 3;
    for (size_t i = 0; i < batch; ++i) {
        sizes[i] = static_cast<size_t>(g_ws.sizes_host[i]) + g * 1024;
        bounds[i] = g_ws.ebs_host[i];
    }
    return cudaGetLastError() == cudaSuccess ? 0 : 4;
}

// Decompress `batch` pages.  mode 0: contiguous [batch][n] into dest[0];
// mode 1: scatter into dest[page * per_page + d] of `elements_per_dest`
// each; mode 2: layer-indexed scatter into dest[page].  Asynchronous on the
// stream, like the wrapper's decompress methods.
int ref_decompress_bf16(const unsigned char* const* inputs, size_t batch,
                        size_t n, const float* bounds, int mode,
                        void* const* dest, size_t per_page,
                        size_t elements_per_dest,
                        const int64_t* layer_indices, size_t selected,
                        size_t prefix_count, size_t source_layers,
                        size_t elements_per_layer, void* stream_ptr) {
    cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
    size_t logical = mode == 2 ? prefix_count * selected * elements_per_layer
                               : n;
    size_t g = groups_of(logical);
    size_t entries = (g + 1) * batch;
    size_t dest_count = mode == 1 ? batch * per_page : batch;
    if (!g_ws.reserve(entries, dest_count > batch ? dest_count : batch, batch))
        return 1;
    cudaMemcpyAsync(g_ws.ptrs_a, inputs, batch * sizeof(void*),
                    cudaMemcpyHostToDevice, stream);
    cudaMemcpyAsync(g_ws.ebs, bounds, batch * 4, cudaMemcpyHostToDevice,
                    stream);
    g_ws.zero(entries, stream);
    bool ok;
    auto cmp = reinterpret_cast<const unsigned char* const*>(g_ws.ptrs_a);
    if (mode == 0) {
        ok = launch_cuszp_decompress_batch_fixed_bf16(
            dest[0], cmp, g_ws.cmp, g_ws.local, g_ws.flags, g_ws.ebs, n,
            batch, stream);
    } else {
        cudaMemcpyAsync(g_ws.ptrs_b, dest, dest_count * sizeof(void*),
                        cudaMemcpyHostToDevice, stream);
        if (mode == 1) {
            ok = launch_cuszp_decompress_batch_fixed_bf16_scatter(
                g_ws.ptrs_b, per_page, elements_per_dest, cmp, g_ws.cmp,
                g_ws.local, g_ws.flags, g_ws.ebs, n, batch, stream);
        } else {
            ok = launch_cuszp_decompress_batch_fixed_bf16_indexed_scatter(
                g_ws.ptrs_b, cmp, g_ws.cmp, g_ws.local, g_ws.flags, g_ws.ebs,
                layer_indices, prefix_count, source_layers,
                elements_per_layer, selected, batch, stream);
        }
    }
    if (!ok) return 2;
    return cudaGetLastError() == cudaSuccess ? 0 : 4;
}

}  // extern "C"
