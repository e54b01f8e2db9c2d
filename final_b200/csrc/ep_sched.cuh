// ep_sched.cuh -- the fused expert-parallel pipeline's group lists in owner
// placement, as one __host__ __device__ function: the GPU runs it (one
// thread, the count matrix in shared memory) to start W1||W3 without waiting
// for the host, and the host runs the same code for the copies it issues
// (dispatch sizes, return chunks), so both sides agree by construction.
//
// Owner placement (rank r holds experts [r*EL, (r+1)*EL), EL = E/G), from
// the [G][E] count matrix cnt (rows of source s routed to expert e):
//   within(s, e) = sum of cnt[s][e'] over r's experts e' < e
//   recv_off(s)  = rows of sources s' < s for r's experts (receive layout)
//   seg_off(s,e) = recv_off(s) + within(s, e)           (the row's receive row)
//   home(s, e)   = sum_{e' < r*EL} cnt[s][e'] + within(s, e)
//                                                      (its expert-sorted row at s)
// which is the owner branch of b2_ep_plan_compute restated per (source, expert).
#pragma once
#include <cstdint>

namespace b2 {

constexpr int kFusedSchedArrays = 8;  // counts | C rows | tiles | expert | A rows | source | dest | chunk
constexpr int64_t kReturnChunkRows = 4096;
constexpr int kSchedTileRows = 256;   // rows of the CTA-pair GEMM's m-tiles

// A return chunk of the fused pipeline: consecutive W2 groups of one source,
// receive-layout rows [row, row+rows) of out_recv, sent to rows [home,
// home+rows) of the source's sout once its counter reaches `target`.
struct ReturnChunk {
  int src;
  int64_t row, home, rows;
  uint64_t target;  // epilogue-warp completions of the chunk's tiles
};

// Group list of one fused launch of rank r (w2 = false: W1||W3, true: W2)
// into h (kFusedSchedArrays arrays of n1 = max groups + 1 ints), with the
// same order and chunking as the plan-based builder in ep.cu:
//   W1||W3: sources r, r-1, r-2, ...; A = the own rows in place (sorted_x at
//           home) or a peer's rows in the receive buffer (seg_off, behind its
//           flag); C = seg_off of the intermediate;
//   W2:     sources r-1, r-2, ..., then r; A = seg_off; C = home in sout for
//           the own rows, seg_off in the results buffer for a peer's rows,
//           which form return chunks of ~kReturnChunkRows rows.
// Returns the number of groups (-1 if more than n1 - 1); *mtiles the
// 256-row tiles; chunks / nchunks (may be null) the return chunks with their
// counter targets for W2's n_tiles output tiles per row block.
__host__ __device__ inline int owner_fused_schedule(int G, int r, int E, const int32_t *cnt,
                                                    bool w2, int n_tiles, int n1, int32_t *h,
                                                    int *mtiles, ReturnChunk *chunks,
                                                    int *nchunks) {
  const int EL = E / G, e0 = r * EL;
  int32_t *hc = h, *ho = h + n1, *hm = h + 2 * n1, *hg = h + 3 * n1, *ha = h + 4 * n1,
          *hs = h + 5 * n1, *hd = h + 6 * n1, *hk = h + 7 * n1;
  int n = 0, mt = 0, nch = 0;
  for (int k = 0; k < G; ++k) {
    const int src = w2 ? (k < G - 1 ? (r - 1 - k + 2 * G) % G : r) : (r - k + G) % G;
    const int32_t *cs = cnt + (int64_t)src * E;
    int64_t recv_off = 0;  // rows of the sources before src, for r's experts
    for (int s = 0; s < src; ++s)
      for (int e = e0; e < e0 + EL; ++e) recv_off += cnt[(int64_t)s * E + e];
    int64_t before = 0;  // src's rows of the experts before r's
    for (int e = 0; e < e0; ++e) before += cs[e];
    ReturnChunk cur{-1, 0, 0, 0, 0};
    int64_t within = 0;
    for (int el = 0; el < EL; ++el) {
      const int32_t c = cs[e0 + el];
      if (c == 0) continue;
      if (n >= n1 - 1) return -1;
      const int64_t seg_off = recv_off + within, home = before + within;
      within += c;
      const int tiles = (c + kSchedTileRows - 1) / kSchedTileRows;
      hc[n] = c;
      hg[n] = el;
      hk[n] = -1;
      if (!w2) {
        ho[n] = (int32_t)seg_off;
        ha[n] = (int32_t)(src == r ? home : seg_off);
        hs[n] = src == r ? -1 : src;
        hd[n] = 0;
      } else {
        ho[n] = (int32_t)(src == r ? home : seg_off);
        ha[n] = (int32_t)seg_off;
        hs[n] = -1;
        hd[n] = src;
        if (src != r) {
          if (cur.src < 0 || cur.rows >= kReturnChunkRows || cur.row + cur.rows != seg_off) {
            if (cur.src >= 0) {
              if (chunks) chunks[nch] = cur;
              ++nch;
            }
            cur = ReturnChunk{src, seg_off, home, 0, 0};
          }
          cur.rows += c;
          cur.target += 8ull * (uint64_t)tiles * (uint64_t)n_tiles;  // 8 epilogue warps per tile
          hk[n] = nch;
        }
      }
      hm[n] = mt;
      mt += tiles;
      ++n;
    }
    // within a source, the owned experts' rows are contiguous, so a source's
    // consecutive groups always continue the open chunk unless it is full
    if (cur.src >= 0) {
      if (chunks) chunks[nch] = cur;
      ++nch;
    }
  }
  hm[n] = mt;
  *mtiles = mt;
  if (nchunks) *nchunks = nch;
  return n;
}

}  // namespace b2
