/*
 * b2mlp.h -- dense SwiGLU MLP (the feed-forward block of the layers without
 * experts) on the same tcgen05 GEMM core as the MoE experts (C ABI).
 *
 *   y[T, H] = (silu(x . W1^T) * (x . W3^T)) . W2^T
 *
 * W1 (gate, silu applied) and W3 (up) are [inter][hidden], W2 is
 * [hidden][inter], fp32 row-major, as the reference stores them.  Replaces
 * MLP::init_gpu / MLP::forward_gpu (include/layer.h:48-66,
 * src/layer.cu:1217-1269): there three attn_matmul_tiled_kernel launches and
 * moe_swiglu_kernel (src/layer.cu:670-692); here W1||W3 + SwiGLU is one
 * GEMM with the gating in its epilogue and W2 a second one writing y.
 *
 * The reference forward never allocates its temp_buf_gpu_ (the allocation
 * branch at src/layer.cu:1232 is empty); this object owns all its scratch.
 */
#ifndef B2MLP_H
#define B2MLP_H

#include "b2moe.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct b2_mlp_desc {
  int hidden;     /* H, multiple of 8 (reference: 2048, include/config.h) */
  int inter;      /* I, any >= 1 (padded internally to 128; reference 7168) */
  int max_tokens; /* scratch capacity in tokens */
  int dtype;      /* B2_BF16 or B2_TF32 */
} b2_mlp_desc;

typedef struct b2_mlp b2_mlp;

/* Packs the weights (device or host fp32 pointers, see weights_on_host) and
 * allocates scratch for max_tokens tokens.  Synchronises `stream` once. */
b2_status b2_mlp_create(const b2_mlp_desc *desc, const float *w1, const float *w2,
                        const float *w3, int weights_on_host, b2_stream stream,
                        b2_mlp **out);

/* y[T,H] = MLP(x[T,H]); x, y device fp32 row-major.  Stream-ordered, no host
 * synchronisation.  B2_ERR_CAPACITY if num_tokens > max_tokens. */
b2_status b2_mlp_forward(b2_mlp *mlp, const float *x, float *y, int num_tokens,
                         b2_stream stream);

/* Synchronises `stream`, returns and clears the device status word. */
b2_status b2_mlp_get_status(b2_mlp *mlp, b2_stream stream, int *device_status);

/* Bytes of device memory the object holds. */
size_t b2_mlp_device_bytes(const b2_mlp *mlp);

b2_status b2_mlp_destroy(b2_mlp *mlp);

#ifdef __cplusplus
}
#endif

#endif /* B2MLP_H */
