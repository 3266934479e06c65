// Shared between the two varlen prefill kernels (mma.sync in flash_prefill.cu, tcgen05 in
// flash_prefill_tc.cu): launch parameters and the device-side query-tile numbering.
#pragma once

#include "common.cuh"

namespace mvb {

struct FaParams {
  const void *q, *k, *v;
  void* o;
  const int32_t* cu;
  int64_t sq_t, sq_h, sk_t, sk_h, sv_t, sv_h, so_t, so_h;
  // paged K/V (paged prefill): k/v are the caches [NB, bs, Hkv, D]; strides sk_b/sk_t/sk_h
  const int32_t* bt;
  const int32_t* ctx;
  int64_t sk_b, sv_b, sbt_s, sbt_b;
  int block_size;
  int n_seqs, hq, hkv, causal;
  float scale_log2;
};

// tcgen05 path: returns -1 when the shape/layout is outside what it handles (the caller then
// runs the mma.sync kernel; *why names the reason), else an MVB status.  T = query tokens,
// n_blocks = cache blocks.
int launch_fa_tc(const FaParams& p, int dtype, int d, bool paged, int64_t T, int64_t n_tokens_kv,
                 int64_t n_blocks, cudaStream_t st, const char** why);

namespace {

// Query tile index -> (sequence, first query of the tile), BM_ queries per tile.  Tiles of
// each sequence are numbered last-first, so under a causal mask the most expensive tiles
// of a sequence launch first.  Every thread of the block must call it.
template <int BM_>
__device__ __forceinline__ bool map_query_tile(const int32_t* cu, int n_seqs, int tile_idx, int& seq, int& q0) {
  __shared__ int s_seq, s_q0;
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    int base = 0, found = -1, fq = 0;
    for (int s0 = 0; s0 < n_seqs && found < 0; s0 += 32) {
      const int s = s0 + lane;
      int cnt = 0;
      if (s < n_seqs) cnt = (cu[s + 1] - cu[s] + BM_ - 1) / BM_;
      int incl = cnt;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      const int excl = base + incl - cnt;
      const bool hit = s < n_seqs && tile_idx >= excl && tile_idx < excl + cnt;
      const unsigned m = __ballot_sync(0xffffffffu, hit);
      if (m) {
        const int src = __ffs(m) - 1;
        found = __shfl_sync(0xffffffffu, s, src);
        fq = __shfl_sync(0xffffffffu, (cnt - 1 - (tile_idx - excl)) * BM_, src);
      }
      base += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) {
      s_seq = found;
      s_q0 = fq;
    }
  }
  __syncthreads();
  seq = s_seq;
  q0 = s_q0;
  return seq >= 0;
}

}  // namespace
}  // namespace mvb
