// Work decomposition shared by the persistent tcgen05 grouped GEMMs: the segment
// table (expert, activation row, output row, row count) and its tile prefix are
// staged in shared memory once per CTA; work item w = (token tile, 128-feature
// tile) is decoded from them with shared-memory reads only.
#pragma once

#include "gemq_internal.h"

namespace gemq {
namespace tcw {

constexpr int kTileN = 128;    // output features per work item (UMMA M)
constexpr int kMaxSegs = 256;  // segments whose metadata every CTA stages
constexpr int kMetaBytes = kMaxSegs * 16 + (kMaxSegs + 1) * 4 + kMaxSegs * 4 * 5 + 16;

struct Work {
  int e, act_row, out_row, rows, n0, nb, wrow0, srow0, wrow1, srow1;
};

struct Meta {
  Seg seg[kMaxSegs];
  int tp[kMaxSegs + 1];
  int nb[kMaxSegs], wrow0[kMaxSegs], srow0[kMaxSegs], wrow1[kMaxSegs], srow1[kMaxSegs];
};
static_assert(sizeof(Meta) <= kMetaBytes, "metadata layout");

// Args provides: tile_prefix, segs, num_segs, nbits, wq_strides0/1, zs_strides0/1, N.
template <class Args>
__device__ __forceinline__ void stage_meta(Meta& m, const Args& p, bool dense) {
  for (int i = threadIdx.x; i <= p.num_segs; i += blockDim.x) m.tp[i] = __ldg(p.tile_prefix + i);
  for (int i = threadIdx.x; i < p.num_segs; i += blockDim.x) {
    const Seg sg = __ldg(p.segs + i);
    m.seg[i] = sg;
    if (dense) {
      m.nb[i] = 4;
      m.wrow0[i] = m.srow0[i] = m.wrow1[i] = m.srow1[i] = 0;
    } else {
      const int e = sg.x;
      m.nb[i] = __ldg(p.nbits + e);
      m.wrow0[i] = __ldg(p.wq_strides0 + e) / p.N;
      m.srow0[i] = __ldg(p.zs_strides0 + e) / p.N;
      m.wrow1[i] = __ldg(p.wq_strides1 + e) / p.N;
      m.srow1[i] = __ldg(p.zs_strides1 + e) / p.N;
    }
  }
}

// Segment of tile t: the last segment whose tile prefix is <= t (binary search).
__device__ __forceinline__ int seg_of_tile(const Meta& m, int num_segs, int t) {
  int lo = 0, hi = num_segs;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (m.tp[mid] <= t) lo = mid; else hi = mid;
  }
  return lo;
}

// Work item w of segment lo (the segment of its token tile).
template <int NT>
__device__ __forceinline__ Work work_in_seg(const Meta& m, int lo, int n_tiles, int w) {
  Work wk;
  const int t = w / n_tiles;
  const int i = w - t * n_tiles;
  const Seg sg = m.seg[lo];
  const int j = t - m.tp[lo];
  wk.e = sg.x;
  wk.act_row = sg.y + j * NT;
  wk.out_row = sg.z + j * NT;
  wk.rows = min(NT, sg.w - j * NT);
  wk.n0 = i * kTileN;
  wk.nb = m.nb[lo];
  wk.wrow0 = m.wrow0[lo];
  wk.srow0 = m.srow0[lo];
  wk.wrow1 = m.wrow1[lo];
  wk.srow1 = m.srow1[lo];
  return wk;
}

template <int NT>
__device__ __forceinline__ Work decode_work(const Meta& m, int num_segs, int n_tiles, int w) {
  return work_in_seg<NT>(m, seg_of_tile(m, num_segs, w / n_tiles), n_tiles, w);
}

}  // namespace tcw
}  // namespace gemq
