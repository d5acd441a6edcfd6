// Host-side launch interface between the C-ABI layer and the kernels.
#pragma once

#include <cuda_runtime.h>
#include <cstdint>

#include "ckv_device.cuh"

namespace ckv {

enum class ElemType { kBF16 = 0, kF32 = 1 };

struct EncodeLaunch {
    const Unit* units;         // device
    const Map* maps;           // device
    uint32_t num_units;
    uint32_t max_n;            // largest unit (elements)
    bool relative;
    uint64_t* sizes;           // device-visible, one per unit
    float* bounds;             // device-visible, one per unit
    uint32_t* status;          // device-visible, one per unit
    ElemType type;
    // Every unit a whole page: identity element map, elements 16-byte
    // aligned, n > 0 (BF16 batches like this may use the streaming encoder).
    bool whole_pages;
    // 0 automatic, 1 clustered encoder, 2 streaming encoder (whole pages only)
    int encoder;
    // Failure-path test hook (0: off): the cluster that owns unit
    // withhold_unit never completes that unit's bound exchange, and its
    // waits give up after test_polls polls (kErrTimeout on its units).
    uint32_t withhold_unit;
    uint32_t test_polls;
};

struct DecodeLaunch {
    const Unit* units;         // device
    const Map* maps;           // device
    uint32_t num_units;
    uint32_t max_n;
    bool zero_fill;            // write rate-0 blocks (the reference skips them)
    uint32_t* status;          // device-visible, one per unit
    ElemType type;             // destination element type
    uint32_t total_items;      // sum of decode_items(unit.n)
    uint32_t uniform_items;    // items per unit if all units have the same n, else 0
};

struct PackUnit {
    const uint8_t* src;
    uint64_t size;
    uint64_t offset;           // byte offset in the destination slab
};

// One page of the INT8 codec: the page (BF16, n elements) and its stored
// form (n int8 values, FP32 scale at byte align4(n)).  amax is a zeroed
// device word the encoder folds the page's max |x| into.
struct Int8Unit {
    const void* page;
    uint8_t* q;
    uint32_t* amax;
    uint32_t n;
    uint32_t pad;
};

// One byte copy.
struct CopyUnit {
    const uint8_t* src;
    uint8_t* dst;
    uint64_t bytes;
};

__host__ __device__ constexpr uint32_t align4(uint32_t x) { return (x + 3u) & ~3u; }

// Work items (256 blocks each) of a unit of n elements in the decoder.
uint32_t decode_items(uint32_t n);

// Largest unit (elements) the single-pass clustered encoder accepts.
uint32_t encode_max_elements(ElemType type);

// Loads every encoder kernel of an element type on the current device (no
// launch); the first launch of a kernel would otherwise load it then.
cudaError_t encode_prepare(ElemType type);

// Enqueue on `stream`; returns cudaSuccess or the launch error.
cudaError_t launch_encode(const EncodeLaunch& l, cudaStream_t stream);
cudaError_t launch_decode(const DecodeLaunch& l, cudaStream_t stream);
cudaError_t launch_pack(const PackUnit* units, uint32_t count, uint64_t max_size,
                        uint8_t* dst, cudaStream_t stream);
// INT8 codec: page max then quantise (two launches), or dequantise.
cudaError_t launch_int8_encode(const Int8Unit* units, uint32_t count, uint32_t max_n,
                               cudaStream_t stream);
cudaError_t launch_int8_decode(const Int8Unit* units, uint32_t count, uint32_t max_n,
                               cudaStream_t stream);
// Byte copies (raw page gather / scatter).
cudaError_t launch_copy(const CopyUnit* units, uint32_t count, uint64_t max_bytes,
                        cudaStream_t stream);
// Copies `bytes` (a multiple of 16, both addresses 16-byte aligned) from
// mapped page-locked host memory to device memory with a kernel.
cudaError_t launch_fetch(const void* mapped_src, void* dst, size_t bytes, cudaStream_t stream);

// Kernel launches made since load (tests and bench count them).
uint64_t launches_issued();
void note_launch();

}  // namespace ckv
