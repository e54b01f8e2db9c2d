/*
 * b2moe.h -- C ABI of the B200-native (sm_100a) MoE / dense-GEMM hot path.
 *
 * Plain pointers and sizes only.  Every call is stream-ordered on the stream
 * it is given and never synchronises the host unless its comment says so.
 * Calls return a b2_status and never exit the process.  Device-side faults
 * that the kernels detect themselves (a bounded wait that expired, an expert
 * id out of range) are recorded in a per-object device status word that
 * b2_moe_get_status() reads.
 *
 * The entry points replace the reference engine's interfaces as noted beside
 * each declaration (paths are within the reference project).
 */
#ifndef B2MOE_H
#define B2MOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st *b2_stream; /* = cudaStream_t */

typedef enum b2_status {
  B2_OK = 0,
  B2_ERR_INVALID = 1,     /* bad argument / unsupported shape */
  B2_ERR_CUDA = 2,        /* a CUDA runtime / driver call failed */
  B2_ERR_CAPACITY = 3,    /* num_tokens > max_tokens of the object */
  B2_ERR_DEVICE = 4,      /* a kernel recorded a device-side error */
  B2_ERR_NO_DEVICE = 5,   /* no sm_100 device present */
  B2_ERR_COMM = 6,        /* collective failed or a peer did not answer in time */
} b2_status;

typedef enum b2_dtype {
  B2_BF16 = 0, /* bf16 operands, fp32 accumulate (tcgen05 kind::f16) */
  B2_TF32 = 1, /* fp32 operands read as TF32, fp32 accumulate (kind::tf32) */
  B2_F32 = 2,  /* fp32 storage (outputs) */
} b2_dtype;

/* Shape and options of one MoE layer.  Defaults of the reference model:
 * hidden 2048, inter 1792, experts 32, top_k 4, routed_scale 1.0, use_bias 1
 * (include/config.h:6,14-20). */
typedef struct b2_moe_desc {
  int hidden;         /* H, multiple of 64 */
  int inter;          /* I, multiple of 16 (padded internally to 128) */
  int num_experts;    /* E, 1..32 */
  int top_k;          /* K, 1..8, <= E */
  int max_tokens;     /* scratch capacity in tokens */
  float routed_scale; /* multiplies the renormalised weights */
  int use_bias;       /* add expert_bias to the selection score */
  int dtype;          /* B2_BF16 or B2_TF32 for the expert GEMMs */
} b2_moe_desc;

typedef struct b2_moe b2_moe;

/* Optional device buffers a forward copies its intermediates into (any may be
 * NULL).  Shapes: logits [T,E] f32; topk_idx [T,K] i32; topk_w [T,K] f32;
 * counts/offsets [E] i32; mtile_offsets [E+1] i32; token_slot [T,K] i32;
 * sorted_token [T*K] i32; sorted_w [T*K] f32. */
typedef struct b2_moe_trace {
  float *logits;
  int32_t *topk_idx;
  float *topk_w;
  int32_t *counts;
  int32_t *offsets;
  int32_t *mtile_offsets;
  int32_t *token_slot;
  int32_t *sorted_token;
  float *sorted_w;
} b2_moe_trace;

/* Replaces SparseMoeBlock::SparseMoeBlock + init_gpu
 * (include/layer.h:74-79, src/layer.cu:1274-1300, 1357-1426).
 * w1, w3: E pointers to fp32 [I,H] row-major; w2: E pointers to fp32 [H,I]
 * (the reference's per-expert float** tables, src/layer.cu:1377-1396).
 * gate: fp32 [E,H]; bias: fp32 [E] or NULL.  weights_on_host != 0 means all
 * of these are host pointers, else device pointers on the current device.
 * Packs the weights into the kernels' layouts, allocates the scratch for
 * desc->max_tokens and synchronises `stream` before returning. */
b2_status b2_moe_create(const b2_moe_desc *desc, const float *const *w1,
                        const float *const *w2, const float *const *w3,
                        const float *gate, const float *bias,
                        int weights_on_host, b2_stream stream, b2_moe **out);

/* Replaces SparseMoeBlock::~SparseMoeBlock (src/layer.cu:1302-1355). */
b2_status b2_moe_destroy(b2_moe *moe);

/* Replaces SparseMoeBlock::forward_gpu(x, y, batch, seq_len, hidden, stream)
 * (include/layer.h:80-81, src/layer.cu:1428-1498): y[T,H] = MoE(x[T,H]),
 * both fp32 device pointers, T = batch*seq_len <= max_tokens. */
b2_status b2_moe_forward(b2_moe *moe, const float *x, float *y, int num_tokens,
                         b2_stream stream);

/* Same as b2_moe_forward, also copying intermediates into `trace`. */
b2_status b2_moe_forward_ex(b2_moe *moe, const float *x, float *y,
                            int num_tokens, const b2_moe_trace *trace,
                            b2_stream stream);

/* Routing step without any device allocation, for callers that may not call
 * cudaMalloc after start-up (a server that plans all device memory up front,
 * or a host whose allocator is owned elsewhere).  No counterpart in the
 * reference: it is the route / scan / slot part of b2_moe_forward on caller
 * buffers, with its scratch in a fixed 1 MiB __device__ array that every GPU
 * loading this library holds until exit.
 * x [T,H] f32, gate [E,H] f32, bias [E] f32 or NULL (device pointers);
 * outputs topk_idx/topk_w/token_slot [T,K], counts/offsets [E].
 * Limits: T > 65536 or H > 4096 return B2_ERR_CAPACITY (the fixed scratch is
 * sized for them); H not a multiple of 64, E outside 1..32, K outside 1..8 or
 * above E, a NULL required pointer or an x that is not 16-byte aligned
 * return B2_ERR_INVALID, all before any device work.  The first call on a
 * device looks up the array's device address (cudaGetSymbolAddress) with
 * that device current; make that first call before any stream capture.  The
 * address is kept for the life of the process, so a cudaDeviceReset (which
 * unloads the module) leaves this entry point unusable on that device.  All
 * calls share the array: calls that overlap on the GPU race and must not be
 * issued. */
b2_status b2_moe_route_noalloc(const float *x, const float *gate,
                               const float *bias, int num_tokens, int hidden,
                               int num_experts, int top_k, float routed_scale,
                               int32_t *topk_idx, float *topk_w,
                               int32_t *counts, int32_t *offsets,
                               int32_t *token_slot, b2_stream stream);

/* Slot bookkeeping of the scatter for expert ids the caller computed itself
 * (e.g. with a router of its own): per-expert counts and offsets and the
 * token -> slot map in the canonical token-major order, on the object's
 * scratch (no allocation).  Replaces moe_scan_kernel and the slot part of
 * moe_scatter_kernel (src/layer.cu:730-768, 501-542) run on a router's
 * output.  topk_idx [T,K] i32 and token_slot [T,K] i32 are device pointers,
 * T <= max_tokens; counts / offsets ([E] i32, device) may be NULL.  An id of
 * -1 means "no expert" and gets slot -1; an id outside [-1, E) also gets slot
 * -1 and is recorded as device status 0x201 (read with b2_moe_get_status),
 * so a corrupt id never addresses memory.  No counterpart of its own in the
 * reference, whose scatter assumes valid ids (src/layer.cu:515-523). */
b2_status b2_moe_dispatch_slots(b2_moe *moe, const int32_t *topk_idx,
                                int num_tokens, int32_t *counts,
                                int32_t *offsets, int32_t *token_slot,
                                b2_stream stream);

/* Synchronises `stream`, returns the device status word (0 = ok) in
 * *device_status and clears it.  B2_ERR_DEVICE when it was non-zero. */
b2_status b2_moe_get_status(b2_moe *moe, b2_stream stream, int *device_status);

/* Stage timing aid for benchmarks.  While enabled, every forward records a
 * CUDA event before each of its six stages and one after the last, on the
 * forward's own stream. */
b2_status b2_moe_profile_enable(b2_moe *moe, int enable);

/* Synchronises on the recorded events and returns the summed milliseconds
 * per stage (route, scan, scatter, gemm_w13, gemm_w2, combine) over the
 * forwards recorded since the last read, and how many there were; clears the
 * record. */
b2_status b2_moe_profile_read(b2_moe *moe, float *stage_ms, int *forwards);

/* Rows per m-tile of the expert GEMMs' schedule (the unit of
 * b2_moe_trace.mtile_offsets). */
int b2_moe_tile_rows(void);

/* Bytes of device memory the object holds (weights + scratch). */
size_t b2_moe_device_bytes(const b2_moe *moe);

/* Dense NT GEMM on the tcgen05 core: C[M,N] (fp32, row stride ldc) =
 * A[M,K] . B[N,K]^T, A and B row-major with row stride K.
 * dtype = B2_BF16: A, B are bf16;  B2_TF32: A, B are fp32 (TF32 math).
 * Replaces attn_matmul_tiled_kernel (src/layer.cu:9-141) at its call sites
 * (src/layer.cu:1250-1268, 1617-1631, 1669-1672, 1747-1756, 1774-1777) and
 * lm_head_gemm_kernel / the cuBLAS fp16 branch (src/model.cu:42-116,
 * 497-548).  K multiple of 8 (bf16) or 4 (tf32); ldc >= N.
 * `status` (device int, may be NULL) receives device-side errors. */
b2_status b2_gemm_nt(const void *A, const void *B, float *C, int M, int N,
                     int K, int ldc, int dtype, int *status, b2_stream stream);

/* b2_gemm_nt with the kernel configuration chosen by the caller instead of
 * the planner (tuning sweeps, tests that reach every kernel on one shape):
 * kind 0 single-CTA tiles of width bn (64, 128, 256); 1 CTA pairs
 * (256 x 256); 2 split-K clusters of `split` CTAs (2..8) over 128 x bn tiles
 * (bn 128 or 256); 3 split-K clusters of `split` CTA pairs (2..4) over
 * 256 x 256 tiles (bn ignored).  No counterpart in the reference. */
b2_status b2_gemm_nt_config(const void *A, const void *B, float *C, int M, int N,
                            int K, int ldc, int dtype, int kind, int bn, int split,
                            int *status, b2_stream stream);

/* The kernel configuration b2_gemm_nt uses for an M x N x K product on a
 * device with `sms` SMs (host only, no device call): *kind = 0 single-CTA
 * tiles, 1 CTA pairs (256 x 256), 2 split-K clusters, 3 split-K clusters of
 * CTA pairs; *bn = output tile width; *split = K-slices per tile (CTAs for
 * kind 2, CTA pairs for kind 3; 1 otherwise).  No
 * counterpart in the reference, whose GEMM has one fixed 128 x 128 tiling
 * (src/layer.cu:9-141). */
b2_status b2_gemm_plan(int M, int N, int K, int dtype, int sms, int *kind, int *bn,
                       int *split);

/* fp32 -> bf16 (round to nearest even), n elements, device pointers. */
b2_status b2_convert_f32_to_bf16(const float *in, void *out, size_t n,
                                 b2_stream stream);

/* Number of kernels of this library launched so far in this process (all
 * devices); lets callers count launches inside a timed region. */
uint64_t b2_kernel_launch_count(void);

const char *b2_status_string(b2_status s);

/* Library build identification string. */
const char *b2_version(void);

/* The architecture the library's device code was compiled for, as the CUDA
 * runtime reports it for one of the library's kernels on the current device
 * (cudaFuncGetAttributes binaryVersion: major * 10 + minor, 100 for sm_100a).
 * Needs a device; B2_ERR_CUDA when the kernel cannot be loaded on it.  No
 * counterpart in the reference. */
b2_status b2_device_code_version(int *version);

#ifdef __cplusplus
}
#endif

#endif /* B2MOE_H */
