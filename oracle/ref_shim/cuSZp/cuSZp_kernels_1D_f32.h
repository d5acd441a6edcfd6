/*
 * Stand-in for upstream cuSZp/cuSZp_kernels_1D_f32.h.  The reference's
 * batched kernels use only the two launch-geometry constants from it
 * (cuszp_batched_fixed.cu:4,164-165,399-402).  Their values follow from the
 * reference itself: one warp per CUDA block (lane = threadIdx.x with
 * full-mask shuffles and lane 31 as the last lane, cuszp_batched_fixed.cu:
 * 162,234-241) and 32 * 1024 elements per CUDA block (kElementsPerBlock,
 * cuszp_wrapper.cpp:268).
 */
#pragma once
static const int tblock_size = 32;
static const int thread_chunk = 1024;
