/*
 * b2moe_ep.h -- expert-parallel MoE layer over several GPUs of one node
 * (C ABI).  One process per GPU; token rows travel between GPUs as
 * copy-engine writes into the peers' buffers (CUDA IPC over NVLink /
 * NVSwitch), NCCL carries the per-forward count all-gather.
 *
 * No counterpart in the reference for the collective path itself: the
 * reference runs each whole decoder layer on one GPU of a 24-stage pipeline
 * and moves activations with cudaMemcpyAsync peer copies
 * (src/model.cu:235-339, 441-468).  b2_ep_forward replaces
 * SparseMoeBlock::forward_gpu (include/layer.h:80-81) on a rank that holds a
 * shard of the tokens.
 *
 * Placement modes:
 *   B2_EP_OWNER     rank r holds experts [r*E/G, (r+1)*E/G) (E divisible by G)
 *                   and computes every row routed to them;
 *   B2_EP_BALANCED  every rank holds all E experts' weights (705 MB in bf16 for
 *                   the reference model) and computes a contiguous share of
 *                   the globally expert-sorted rows (expert-major, then source
 *                   rank), which removes the load imbalance of skewed (e.g.
 *                   Zipf) routing.  Shares split the estimated GEMM cost
 *                   evenly: rows, plus 128 rows' worth per non-empty (expert,
 *                   source) block (a row segment with a partly filled tile)
 *                   and 320 per expert (its weight reads); each rank keeps
 *                   between 1/2 and 3/2 of the mean rows.
 * Both produce bit-identical y to the single-GPU b2_moe_forward on the same
 * tokens: every row goes through the same kernels in the same order.
 */
#ifndef B2MOE_EP_H
#define B2MOE_EP_H

#include "b2moe.h"

#ifdef __cplusplus
extern "C" {
#endif

#define B2_EP_MAX_WORLD 64
#define B2_EP_MAX_SEGMENTS 256
#define B2_EP_UNIQUE_ID_BYTES 128

typedef enum b2_ep_mode { B2_EP_OWNER = 0, B2_EP_BALANCED = 1 } b2_ep_mode;

/* Exchange plan of one rank, computed from the [world][E] matrix of every
 * rank's per-expert row counts.  Row ranges are in units of rows. */
typedef struct b2_ep_plan {
  int64_t send_off[B2_EP_MAX_WORLD]; /* my expert-sorted rows [off, off+cnt) go to rank d */
  int64_t send_cnt[B2_EP_MAX_WORLD];
  int64_t recv_off[B2_EP_MAX_WORLD]; /* rows from rank s land at receive row off */
  int64_t recv_cnt[B2_EP_MAX_WORLD];
  int64_t recv_rows;                 /* total rows this rank computes */
  int32_t num_segments;              /* GEMM row segments of the receive buffer */
  int32_t seg_off[B2_EP_MAX_SEGMENTS];
  int32_t seg_cnt[B2_EP_MAX_SEGMENTS];
  int32_t seg_expert[B2_EP_MAX_SEGMENTS]; /* index into this rank's expert weights */
  int32_t seg_source[B2_EP_MAX_SEGMENTS]; /* rank the segment's rows came from */
} b2_ep_plan;

typedef struct b2_ep b2_ep;

/* Pure host computation (no GPU): the plan of `rank`.  counts is row-major
 * [world][num_experts]. */
b2_status b2_ep_plan_compute(int world, int rank, int num_experts, int mode,
                             const int32_t *counts, b2_ep_plan *plan);

/* NCCL unique id for the communicator (call on rank 0, share the 128 bytes
 * with the other ranks, e.g. through torch.distributed). */
b2_status b2_ep_unique_id(void *id_out);

/* Collective over all ranks.  desc describes the layer as for b2_moe_create
 * (num_experts = all E experts, max_tokens = this rank's token capacity).
 * w1/w2/w3 hold the experts this rank computes: E/world pointers for
 * B2_EP_OWNER (experts rank*E/world ...), all E for B2_EP_BALANCED.  gate and
 * bias are the full router.  Device or host pointers as in b2_moe_create. */
b2_status b2_ep_create(const b2_moe_desc *desc, int world, int rank,
                       const void *unique_id, int mode, const float *const *w1,
                       const float *const *w2, const float *const *w3,
                       const float *gate, const float *bias, int weights_on_host,
                       b2_stream stream, b2_ep **out);

/* Collective.  y[T,H] = MoE(x[T,H]) for this rank's T tokens.  Waits on the
 * host once to size the exchange (the count all-gather, which runs beside the
 * scatter of the rows into expert order); returns
 * B2_ERR_COMM if a peer does not answer within the timeout (the communicator
 * is then aborted).  Rows for rank r+k are pushed by the copy engine into that
 * rank's receive buffer followed by a sequence-number flag; each rank runs its
 * own rows through the expert GEMMs while rows travel, then each source's rows
 * after a bounded wait on its flag (a wait that runs out records a device
 * error readable with b2_moe_get_status on b2_ep_layer) -- in one launch per
 * projection (B2_EP_PIPE_FUSED) or one launch pair per source
 * (B2_EP_PIPE_STAGED) -- and pushes the results back the same way. */
b2_status b2_ep_forward(b2_ep *ep, const float *x, float *y, int num_tokens,
                        b2_stream stream);

/* The bounded device-side wait of the exchange on its own: one thread per
 * flag waits until flags[idx[i]] >= target (device pointers; n <= 1024) and
 * gives up after timeout_s (<= 600) seconds, recording 0x105 in the device
 * int *status (first error wins).  The kernel always returns, so a flag that
 * no peer ever writes leaves the context usable; the caller reads *status
 * after synchronising `stream`.  No counterpart in the reference, whose
 * pipeline stages wait on CUDA events without a bound
 * (src/model.cu:441-445). */
b2_status b2_flag_wait(const uint64_t *flags, const int *idx, int n,
                       uint64_t target, double timeout_s, int *status,
                       b2_stream stream);

/* Marks of the expert-parallel forward's timeline, in stream order. */
enum {
  B2_EP_TL_START = 0,       /* forward entered (before routing) */
  B2_EP_TL_SCATTERED = 1,   /* rows scattered into expert order */
  B2_EP_TL_PLANNED = 2,     /* count matrix on the host, plan made, schedules uploaded */
  B2_EP_TL_OWN_FIRST = 3,   /* first part of the rank's own rows through both GEMMs */
  B2_EP_TL_ARRIVED = 4,     /* one source's rows have arrived (after its flag wait) */
  B2_EP_TL_REMOTE_DONE = 5, /* that source's rows through both GEMMs */
  B2_EP_TL_OWN_SECOND = 6,  /* second part of the own rows through both GEMMs */
  B2_EP_TL_RETURNED = 7,    /* every peer has returned this rank's results */
  B2_EP_TL_DONE = 8,        /* combine done */
  /* host-side durations of the same forward (ms, not times since the first mark) */
  B2_EP_TL_HOST_WAIT = 9,   /* the host's wait for the count matrix */
  B2_EP_TL_HOST_ENQUEUE = 10, /* from that wait's end until the forward returned */
  /* marks of the fused pipeline (B2_EP_PIPE_FUSED) */
  B2_EP_TL_W13_DONE = 11,   /* the one W1||W3 launch over every source's rows */
  B2_EP_TL_W2_DONE = 12     /* the one W2 launch (its chunks' return copies run meanwhile) */
};

/* How a rank runs its expert GEMMs over the rows of every source. */
typedef enum b2_ep_pipeline {
  /* One persistent W1||W3 launch over the rank's own rows and every source's
   * rows (its TMA producer waits, bounded, on each source's arrival flag
   * before loading that source's rows) and one W2 launch over all of them;
   * W2's epilogue counts every stored tile per return chunk (consecutive rows
   * of one source), and the copy engine sends each chunk back to its source
   * as soon as its counter is complete (a 64-bit stream wait on the counter),
   * then raises this rank's flag there.  The default where the device offers
   * 64-bit stream waits. */
  B2_EP_PIPE_FUSED = 0,
  /* One W1||W3 + W2 launch pair per source (own rows split around the remote
   * ones), each remote pair after a flag-wait launch, results returned by
   * copy-engine writes.  Same results, bit for bit. */
  B2_EP_PIPE_STAGED = 1
} b2_ep_pipeline;

/* Selects the pipeline of the following forwards (not collective: every rank
 * may choose its own; the exchange protocol is the same).  B2_ERR_NO_DEVICE
 * for B2_EP_PIPE_FUSED on a device without 64-bit stream waits. */
b2_status b2_ep_set_pipeline(b2_ep *ep, int pipeline);

/* Number of ints of one fused schedule (b2_ep_fused_schedule). */
#define B2_EP_FUSED_SCHED_INTS (8 * (B2_EP_MAX_SEGMENTS + 1))

/* Pure host computation (no GPU): the group list one fused launch of `rank`
 * runs (w2 = 0: W1||W3, w2 != 0: W2), from the [world][E] count matrix (every
 * rank's plan is derived from it as b2_ep_plan_compute does).  sched receives
 * B2_EP_FUSED_SCHED_INTS ints: eight arrays of B2_EP_MAX_SEGMENTS + 1 --
 * row counts; C rows (W1||W3: the receive-layout row of the intermediate;
 * W2: the expert-sorted row in this rank's sout for its own rows, the
 * receive-layout row of the results buffer for a peer's rows); the exclusive
 * prefix of 256-row tiles (one entry more than groups); local expert index;
 * A rows (W1||W3: the own rows' expert-sorted position, the receive-layout
 * row for a peer's rows; W2: the receive-layout row); source rank whose
 * arrival flag a group waits on (-1: none); rank the rows came from; W2's
 * return chunk (-1: none; a chunk is consecutive receive-layout rows of one
 * source, returned to that source's sout in one copy).  *groups and *mtiles:
 * the list's length and tile count.  No counterpart in the reference;
 * exposed so the schedule's row mapping is testable on a CPU. */
b2_status b2_ep_fused_schedule(int world, int rank, int num_experts, int mode,
                               const int32_t *counts, int w2, int32_t *sched,
                               int *groups, int *mtiles);

/* Timeline of the last forward run with profiling on (b2_moe_profile_enable
 * on b2_ep_layer(ep)): *n marks (at most max), tags[i] one of B2_EP_TL_*,
 * ms[i] the device time from the first mark (CUDA events on the forward's
 * stream), followed by the two host durations.  Waits for the last mark.  No
 * counterpart in the reference. */
b2_status b2_ep_profile_timeline(b2_ep *ep, int max, int *tags, float *ms, int *n);

/* Host-side bound (seconds) on every wait for the peers (default 60). */
b2_status b2_ep_set_timeout(b2_ep *ep, double seconds);

/* The plan used by the last forward (for tests and load reports). */
b2_status b2_ep_last_plan(const b2_ep *ep, b2_ep_plan *plan);

/* The single-GPU layer object inside (routing, local scratch, weights);
 * valid until b2_ep_destroy.  Lets callers use b2_moe_profile_* and
 * b2_moe_get_status on the expert-parallel layer. */
b2_moe *b2_ep_layer(b2_ep *ep);

b2_status b2_ep_destroy(b2_ep *ep);

#ifdef __cplusplus
}
#endif

#endif /* B2MOE_EP_H */
