/*
 * Stand-in for the upstream cuSZp public header (szcompressor/cuSZp at
 * f581dcf329c907c320f4743a9c6e7ee2fb9c5494, not vendored by the reference).
 * Only what the reference's cuszp_fastpath.h and cuszp_batched_fixed.cu
 * need to compile: the three enum types it names in prototypes.  Used only
 * to build the reference kernels into oracle/_ref/ as a test oracle.  The
 * values are libckv's (include/ckv.h CKV_DIM_* / CKV_MODE_* / CKV_TYPE_*),
 * which follow the reference's binding order (pybind11_bindings.cpp:13-28).
 */
#pragma once
typedef enum { CUSZP_DIM_1D = 0, CUSZP_DIM_2D = 1, CUSZP_DIM_3D = 2 } cuszp_dim_t;
typedef enum { CUSZP_MODE_FIXED = 0, CUSZP_MODE_PLAIN = 1, CUSZP_MODE_OUTLIER = 2 } cuszp_mode_t;
typedef enum { CUSZP_TYPE_FLOAT = 0, CUSZP_TYPE_DOUBLE = 1 } cuszp_type_t;
