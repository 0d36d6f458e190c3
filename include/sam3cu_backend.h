/*
 * include/sam3cu_backend.h - the CUDA (sm_100a) backend as a drop-in for
 * sam3.c's backend vtable.
 *
 *   const struct sam3_backend_ops *sam3_cuda_backend_ops(void);
 *       replaces nothing: it sits next to sam3_cpu_backend_ops()
 *       (src/backend/cpu/cpu_backend.c:220) and sam3_metal_backend_ops()
 *       and implements struct sam3_backend_ops (src/backend/backend.h:29-56).
 *   struct sam3_cuda_backend
 *       the backend instance, base struct first, as every sam3.c backend
 *       (backend.h:59-62); the factory calloc's sizeof() of it and calls
 *       ops->init (backend.c:36-78).
 *
 * The graph types below mirror sam3.c's field for field (sam3_types.h,
 * core/tensor.h:24-49, core/graph.h:25-103, backend/backend.h:22-62), so a
 * struct sam3_graph built by the reference's own model code (gh_* helpers,
 * sam3_vit_build) is evaluated unchanged.  Inside a sam3.c tree include the
 * reference's headers first: their include guards then skip these mirrors.
 */
#ifndef SAM3CU_BACKEND_H
#define SAM3CU_BACKEND_H

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#include "sam3cu.h"

#ifdef __cplusplus
extern "C" {
#endif

#ifndef SAM3_TYPES_H
#define SAM3_MAX_DIMS 4
enum sam3_error {
	SAM3_OK = 0, SAM3_EINVAL = -1, SAM3_ENOMEM = -2, SAM3_EIO = -3,
	SAM3_EBACKEND = -4, SAM3_EMODEL = -5, SAM3_EDTYPE = -6, SAM3_EVIDEO = -7,
};
enum sam3_dtype {
	SAM3_DTYPE_F32, SAM3_DTYPE_F16, SAM3_DTYPE_BF16, SAM3_DTYPE_I32,
	SAM3_DTYPE_I8, SAM3_DTYPE_Q8_0,
};
#endif

#ifndef SAM3_CORE_TENSOR_H
struct sam3_tensor {
	enum sam3_dtype dtype;
	int             n_dims;
	int             dims[SAM3_MAX_DIMS];
	int             strides[SAM3_MAX_DIMS];
	void           *data;
	size_t          nbytes;
	int             ephemeral;
	int             dbg_force_readback;
};
#endif

#ifndef SAM3_CORE_GRAPH_H
#define SAM3_GRAPH_MAX_NODES 16384
#define SAM3_NODE_MAX_INPUTS 8
enum sam3_op {
	SAM3_OP_NONE, SAM3_OP_MATMUL, SAM3_OP_ADD, SAM3_OP_MUL, SAM3_OP_SOFTMAX,
	SAM3_OP_RELU, SAM3_OP_GELU, SAM3_OP_LAYERNORM, SAM3_OP_CONV2D,
	SAM3_OP_RESHAPE, SAM3_OP_TRANSPOSE, SAM3_OP_CAST, SAM3_OP_CONCAT,
	SAM3_OP_SLICE, SAM3_OP_EMBED, SAM3_OP_SIGMOID, SAM3_OP_UPSAMPLE,
	SAM3_OP_ROPE, SAM3_OP_SILU, SAM3_OP_CONV_TRANSPOSE2D,
	SAM3_OP_MAXPOOL2D, SAM3_OP_SDPA, SAM3_OP_BIAS_ADD, SAM3_OP_GROUPNORM,
	SAM3_OP_BATCHNORM, SAM3_OP_HSWISH, SAM3_OP_DIV, SAM3_OP_COUNT,
};
struct sam3_node {
	enum sam3_op        op;
	struct sam3_tensor *inputs[SAM3_NODE_MAX_INPUTS];
	int                 n_inputs;
	struct sam3_tensor *output;
	int                 params[4];
};
struct sam3_graph {
	struct sam3_node nodes[SAM3_GRAPH_MAX_NODES];
	int              n_nodes;
	bool             no_readback;
};
#endif

#ifndef SAM3_BACKEND_H
enum sam3_backend_type {
	SAM3_BACKEND_CPU,
	SAM3_BACKEND_METAL,
	SAM3_BACKEND_CUDA,
};
struct sam3_backend;
struct sam3_backend_ops {
	enum sam3_error (*init)(struct sam3_backend *be);
	void (*free)(struct sam3_backend *be);
	enum sam3_error (*alloc_tensor)(struct sam3_backend *be,
					struct sam3_tensor *t);
	enum sam3_error (*graph_eval)(struct sam3_backend *be,
				      struct sam3_graph *g);
	void (*arena_reset)(struct sam3_backend *be);
	void (*cache_invalidate)(struct sam3_backend *be, const void *start,
				 size_t len);
};
struct sam3_backend {
	enum sam3_backend_type         type;
	const struct sam3_backend_ops *ops;
};
#endif

/* Value of the new enum sam3_backend_type entry (after CPU and METAL). */
#define SAM3CU_BACKEND_TYPE 2

/*
 * CUDA backend instance.  `device` selects the GPU (the factory leaves it 0;
 * set it before init for another device).  Device state lives behind
 * `impl`.  One instance is used by one host thread at a time, like every
 * sam3.c backend (processor / async text worker contract).
 */
struct sam3_cuda_backend {
	struct sam3_backend base; /* must be first */
	int                 device;
	void               *impl;
};

/*
 * The vtable.
 *   init          selects the device, creates a stream and the caches.
 *   alloc_tensor  fills t->data / nbytes / strides from a HOST buffer of
 *                 the backend (model code reads results from t->data, as on
 *                 the CPU backend; the device copy is made on first use).
 *   graph_eval    lowers every node to device kernels in array order: the
 *                 TRANSPOSE(W) -> MATMUL -> ADD(bias) [-> GELU] chain of
 *                 gh_linear / gh_mlp becomes one fused tcgen05 GEMM, the
 *                 other nodes map one-to-one (MATMUL F32/F16/BF16/F32xQ8_0,
 *                 ADD, GELU, LAYERNORM, ROPE, SDPA, SLICE, RESHAPE (alias),
 *                 TRANSPOSE/PERMUTE, CAST, CONV2D groups 1).  Any other
 *                 (op, dtype) returns SAM3_EDTYPE: there is no CPU fallback.
 *                 Graph inputs are uploaded from t->data (non-ephemeral ones
 *                 once, cached by header address); outputs that no later
 *                 node consumes are copied back to t->data unless
 *                 g->no_readback, in which case they stay cached on device.
 *   arena_reset   drops the host arena and the per-graph device buffers.
 *   cache_invalidate drops cached device copies of tensors whose header or
 *                 data lies in [start, start + len).
 */
SAM3CU_API const struct sam3_backend_ops *sam3_cuda_backend_ops(void);

/* Measurement hook, no counterpart in the reference: with the environment
 * variable SAM3CU_VTABLE_PROFILE=1 set when the backend was created, every
 * graph node is timed with a stream sync around it; this prints the
 * per-op-kind totals (plus uploads and read-backs) to stderr and resets
 * them.  A no-op otherwise. */
SAM3CU_API void sam3cu_backend_profile_dump(struct sam3_backend *be);

#ifdef __cplusplus
}
#endif

#endif /* SAM3CU_BACKEND_H */
