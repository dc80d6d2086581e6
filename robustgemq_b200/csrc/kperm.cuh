// K-order of the decode-batch tensor-core GEMM.
//
// The GEMM consumes K in stages of 128. Inside a stage, MMA slot s (0..127) of both
// operands carries k = k0 + kperm(s): the dequantised weight tile holds, in each
// 32-bit column, two codes that one shift and one mask extract from a packed word
// (16 bits apart), and the activations are stored in the same order by the kernel
// that writes them (dispatch for the gate/up input, the gate/up epilogue for the
// down-projection input). A dot product is a sum over k, so the order of the slots
// changes only the order of the fp32 accumulation.
//
// b in {1, 2, 4}: eps = 32/b codes per word; word i of the stage holds k = i*eps + j;
//   slot 2*(i*eps/2 + j) + h  <->  k = i*eps + j + h*eps/2   (j < eps/2, h in {0, 1}),
//   i.e. code j and code j + eps/2 share a column, one `(w >> b*j) & mask` apart.
// b = 3: ten codes per word (bits 30-31 unused); a stage starts at code slot
//   P = k0 % 10 of its first word (P in {0, 2, 4, 6, 8}, index P/2). Codes j and j+5
//   of one word pair up when both fall in the stage; the rest (at most one partial
//   word at each end) pair in increasing k. The tables below list the pairs.
#pragma once

#include <cstdint>

namespace gemq {
namespace kperm {

constexpr int kStageK = 128;

__host__ __device__ constexpr int perm_pow2(int nb, int s) {
  const int eps = 32 / nb, half = eps / 2;
  return (s / eps) * eps + (s % eps) / 2 + (s % 2) * half;
}
__host__ __device__ constexpr int inv_pow2(int nb, int q) {
  const int eps = 32 / nb, half = eps / 2;
  const int r = q % eps;
  return (q / eps) * eps + 2 * (r % half) + r / half;
}

// One column of a 3-bit stage: kind 0 = codes (sa, sa + 5) of word wa; kind 1 =
// code sa of word wa (low half) and code sb of word wb (high half). qa < qb are
// the stage offsets of the two codes.
struct Pair3 {
  int kind, wa, sa, wb, sb, qa, qb;
};
struct Tab3 {
  Pair3 p[5][64];
  int fwd[5][128];  // slot -> k offset
  int inv[5][128];  // k offset -> slot
};

__host__ __device__ constexpr Tab3 make_tab3() {
  Tab3 t{};
  for (int ph = 0; ph < 5; ++ph) {
    const int P = 2 * ph;
    bool used[128] = {};
    int n = 0;
    for (int wi = 0; wi < 14; ++wi) {
      for (int j = 0; j < 5; ++j) {
        const int qa = 10 * wi + j - P, qb = qa + 5;
        if (qa >= 0 && qb < 128) {
          t.p[ph][n] = Pair3{0, wi, j, wi, j + 5, qa, qb};
          used[qa] = true;
          used[qb] = true;
          ++n;
        }
      }
    }
    int pend = -1;
    for (int q = 0; q < 128; ++q) {
      if (used[q]) continue;
      if (pend < 0) {
        pend = q;
        continue;
      }
      t.p[ph][n] = Pair3{1, (pend + P) / 10, (pend + P) % 10, (q + P) / 10, (q + P) % 10, pend, q};
      ++n;
      pend = -1;
    }
    for (int c = 0; c < 64; ++c) {
      t.fwd[ph][2 * c] = t.p[ph][c].qa;
      t.fwd[ph][2 * c + 1] = t.p[ph][c].qb;
    }
    for (int s = 0; s < 128; ++s) t.inv[ph][t.fwd[ph][s]] = s;
  }
  return t;
}

__host__ __device__ constexpr Pair3 pair3(int ph, int c) { return make_tab3().p[ph][c]; }

// Phase index of stage `st` for 3-bit: (128 st) % 10 / 2.
__host__ __device__ constexpr int phase3(int st) { return ((8 * st) % 10) / 2; }

// Word row offset of stage `st` inside an expert's packed rows.
__host__ __device__ constexpr int stage_word_row(int nb, int st) {
  return nb == 3 ? (kStageK * st) / 10 : st * (kStageK * nb / 32);
}
// Word rows one stage reads.
__host__ __device__ constexpr int stage_word_rows(int nb) { return nb == 3 ? 14 : kStageK * nb / 32; }

struct Perm3 {
  uint8_t fwd[5][128];
  uint8_t inv[5][128];
};
__host__ __device__ constexpr Perm3 make_perm3() {
  const Tab3 t = make_tab3();
  Perm3 p{};
  for (int ph = 0; ph < 5; ++ph)
    for (int s = 0; s < 128; ++s) {
      p.fwd[ph][s] = static_cast<uint8_t>(t.fwd[ph][s]);
      p.inv[ph][s] = static_cast<uint8_t>(t.inv[ph][s]);
    }
  return p;
}

}  // namespace kperm
}  // namespace gemq
