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

// Work items (256 blocks each) of a unit of n elements in the decoder.
uint32_t decode_items(uint32_t n);

// Largest unit (elements) the single-pass clustered encoder accepts.
uint32_t encode_max_elements(ElemType type);

// Enqueue on `stream`; returns cudaSuccess or the launch error.
cudaError_t launch_encode(const EncodeLaunch& l, cudaStream_t stream);
cudaError_t launch_decode(const DecodeLaunch& l, cudaStream_t stream);
cudaError_t launch_pack(const PackUnit* units, uint32_t count, uint64_t max_size,
                        uint8_t* dst, cudaStream_t stream);
// Copies `bytes` (a multiple of 16, both addresses 16-byte aligned) from
// mapped page-locked host memory to device memory with a kernel.
cudaError_t launch_fetch(const void* mapped_src, void* dst, size_t bytes, cudaStream_t stream);

// Kernel launches made since load (tests and bench count them).
uint64_t launches_issued();
void note_launch();

}  // namespace ckv
