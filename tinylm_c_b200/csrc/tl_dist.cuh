// tl_dist.cuh -- the data-parallel pieces the device training step uses.
#pragma once
#include "tl_common.cuh"

namespace tl {

constexpr int kMaxShards = 16;   // ranks the overlapped reduction supports

// State of one step's overlapped gradient reduction (see tl_dist.cu).
struct OverlapState {
  float *G = nullptr;
  size_t n_pad = 0, shard = 0;
  int next = -1;     // highest shard not yet issued
  int events = 0;
};

int overlap_begin(DeviceCtx *c, float *G, size_t n, OverlapState *o);
// G[done_from, n_pad) holds this rank's final gradient: issue the reduction
// of every remaining shard inside that range.
int overlap_ready(DeviceCtx *c, OverlapState *o, size_t done_from);
int overlap_finish(DeviceCtx *c, OverlapState *o);
// Sum of squares, clip, AdamW on the shard and all-gather of P, after
// overlap_finish has left the averaged shard in G.
int zero1_finish_after_overlap(DeviceCtx *c, float *P, float *G, float *M_shard, float *V_shard, size_t n,
                               float lr, float b1, float b2, float wd, int t, float max_norm, float *norm_dev);

}  // namespace tl
