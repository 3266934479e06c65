// Causal depthwise conv1d (width 2 <= W <= 6, as the reference kernel) + SiLU, HBM-bound.
//
// Replaces _causal_conv1d_fwd_kernel / _causal_conv1d_update_kernel
// (m/ops/causal_conv1d.py:6-218, :277-431) with the intended math:
//   xp = concat(conv_state[idx] (W-1 rows), x_seq)
//   out[t, c] = silu(sum_j w[c, j] xp[t + j, c])        (fp32 accumulation)
//   conv_state[idx] <- xp[L : L + W - 1]
//
// Prefill tiling: each CTA owns one tile of tokens that never crosses a sequence boundary
// (tiles are numbered per sequence, so the grid is an upper bound ceil(T/TILE) + S and
// surplus CTAs exit).  The tile holding a sequence's first token is the only reader of its
// old conv state; it also writes the new state (reading the tail of x directly), so there is
// no cross-CTA race on conv_state.
// Fast path (16-bit data, contiguous 16-byte aligned rows): conv1d_fwd_pipe_kernel, 64-token
// tiles, rows streamed through registers in groups of 8 16-byte loads per thread.
// Generic path (fp32, strided or unaligned): one thread per VEC channels reading rows
// directly.
#include "common.cuh"

namespace mvb {
namespace {

constexpr int kMinW = 2;
constexpr int kMaxW = 6;

struct ConvParams {
  const void* x;
  const void* w;
  void* state;
  const int32_t* idx;
  const int32_t* cu;
  void* out;
  int64_t sx_t, sx_c, sw_c, sw_j, ss_n, ss_t, ss_c, so_t, so_c;
  int n_seqs, dim, width, silu, tile;
};

// SiLU for the 16-bit outputs: x sigmoid(x) = 0.5 x (1 + tanh(x / 2)) with the hardware
// tanh.approx.f32 (one MUFU op; its ~2^-11 relative error is well below the bf16/fp16
// rounding of the result).
// (6.7% faster than ex2 + fast divide at config 1: the kernel is issue-bound).
__device__ __forceinline__ float silu_fast(float x) {
  const float h = 0.5f * x;
  float t;
  asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(h));
  return fmaf(h, t, h);
}

template <typename T, typename TW, int VEC>
__device__ __forceinline__ void load_vec(const T* base, int64_t stride_c, float* f) {
  if constexpr (VEC == 8) {
    unpack8<T>(*reinterpret_cast<const uint4*>(base), f);
  } else {
#pragma unroll
    for (int i = 0; i < VEC; ++i) f[i] = to_f32<T>(base[i * stride_c]);
  }
}

template <typename T, int VEC>
__device__ __forceinline__ void store_vec(T* base, int64_t stride_c, const float* f) {
  if constexpr (VEC == 8) {
    *reinterpret_cast<uint4*>(base) = pack8<T>(f);
  } else {
#pragma unroll
    for (int i = 0; i < VEC; ++i) base[i * stride_c] = from_f32<T>(f[i]);
  }
}

// Maps tile index -> (seq, first position) using per-sequence tile counts.  One warp
// scans cu_seqlens with a warp-wide prefix sum (S <= a few thousand).
__device__ __forceinline__ bool find_tile(const int32_t* cu, int n_seqs, int tile, int tile_idx, int& seq,
                                          int& pos0) {
  __shared__ int s_seq, s_pos;
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    int base = 0;
    int found = -1, fpos = 0;
    for (int s0 = 0; s0 < n_seqs && found < 0; s0 += 32) {
      const int s = s0 + lane;
      int cnt = 0;
      if (s < n_seqs) cnt = (cu[s + 1] - cu[s] + tile - 1) / tile;
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
        fpos = __shfl_sync(0xffffffffu, (tile_idx - excl) * tile, src);
      }
      base += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) {
      s_seq = found;
      s_pos = fpos;
    }
  }
  __syncthreads();
  seq = s_seq;
  pos0 = s_pos;
  return seq >= 0;
}

template <typename T, typename TW, int VEC, int W>
__global__ void __launch_bounds__(128) conv1d_fwd_kernel(ConvParams p) {
  int seq, pos0;
  if (!find_tile(p.cu, p.n_seqs, p.tile, blockIdx.x, seq, pos0)) return;
  const int c0 = (blockIdx.y * blockDim.x + threadIdx.x) * VEC;
  if (c0 >= p.dim) return;
  const int start = p.cu[seq];
  const int L = p.cu[seq + 1] - start;
  const int pend = min(L, pos0 + p.tile);
  const T* x = static_cast<const T*>(p.x);
  const TW* wp = static_cast<const TW*>(p.w);
  T* st = static_cast<T*>(p.state) + (int64_t)p.idx[seq] * p.ss_n;
  T* out = static_cast<T*>(p.out);

  float w[kMaxW][VEC];
#pragma unroll
  for (int j = 0; j < kMaxW; ++j)
#pragma unroll
    for (int i = 0; i < VEC; ++i) w[j][i] = j < W ? to_f32<TW>(wp[(int64_t)(c0 + i) * p.sw_c + j * p.sw_j]) : 0.f;

  // hist[j] = xp[pos0 + j] for j < W-1  (xp index = position + W-1 maps to x[position])
  float hist[kMaxW - 1][VEC];
#pragma unroll
  for (int j = 0; j < kMaxW - 1; ++j) {
    if (j < W - 1) {
      const int xpi = pos0 + j;  // index into xp
      if (xpi < W - 1)
        load_vec<T, TW, VEC>(st + xpi * p.ss_t + c0 * p.ss_c, p.ss_c, hist[j]);
      else
        load_vec<T, TW, VEC>(x + (int64_t)(start + xpi - (W - 1)) * p.sx_t + c0 * p.sx_c, p.sx_c, hist[j]);
    }
  }

  // New state (only the tile that owns position 0 reads and writes conv_state).
  if (pos0 == 0) {
    float ns[kMaxW - 1][VEC];
#pragma unroll
    for (int j = 0; j < kMaxW - 1; ++j) {
      if (j < W - 1) {
        const int xpi = L + j;
        if (xpi < W - 1) {
#pragma unroll
          for (int jj = 0; jj < kMaxW - 1; ++jj)
            if (jj == xpi)
#pragma unroll
              for (int i = 0; i < VEC; ++i) ns[j][i] = hist[jj][i];
        } else {
          load_vec<T, TW, VEC>(x + (int64_t)(start + xpi - (W - 1)) * p.sx_t + c0 * p.sx_c, p.sx_c, ns[j]);
        }
      }
    }
#pragma unroll
    for (int j = 0; j < kMaxW - 1; ++j)
      if (j < W - 1) store_vec<T, VEC>(st + j * p.ss_t + c0 * p.ss_c, p.ss_c, ns[j]);
  }

  constexpr int B = 8;
  for (int t0 = pos0; t0 < pend; t0 += B) {
    float cur[B][VEC];
#pragma unroll
    for (int b = 0; b < B; ++b)
      if (t0 + b < pend) load_vec<T, TW, VEC>(x + (int64_t)(start + t0 + b) * p.sx_t + c0 * p.sx_c, p.sx_c, cur[b]);
#pragma unroll
    for (int b = 0; b < B; ++b) {
      if (t0 + b < pend) {
        float acc[VEC];
#pragma unroll
        for (int i = 0; i < VEC; ++i) acc[i] = 0.f;
#pragma unroll
        for (int j = 0; j < kMaxW - 1; ++j)
          if (j < W - 1)
#pragma unroll
            for (int i = 0; i < VEC; ++i) acc[i] += w[j][i] * hist[j][i];
#pragma unroll
        for (int j = 0; j < kMaxW; ++j)
          if (j == W - 1)
#pragma unroll
            for (int i = 0; i < VEC; ++i) acc[i] += w[j][i] * cur[b][i];
        if (p.silu)
#pragma unroll
          for (int i = 0; i < VEC; ++i) acc[i] = silu(acc[i]);
        store_vec<T, VEC>(out + (int64_t)(start + t0 + b) * p.so_t + c0 * p.so_c, p.so_c, acc);
        // slide the window
#pragma unroll
        for (int j = 0; j < kMaxW - 2; ++j)
          if (j < W - 2)
#pragma unroll
            for (int i = 0; i < VEC; ++i) hist[j][i] = hist[j + 1][i];
#pragma unroll
        for (int j = 0; j < kMaxW - 1; ++j)
          if (j == W - 2)
#pragma unroll
            for (int i = 0; i < VEC; ++i) hist[j][i] = cur[b][i];
      }
    }
  }
}

// Register-pipelined prefill (16-bit data, contiguous 16-byte rows): a CTA owns kPipeTile
// tokens x 1024 channels, each thread 8 channels; rows stream through registers in groups
// of kPipeDepth, double-buffered (the next group's loads are in flight while this group's
// outputs are computed), the token loop stays rolled so the body fits the instruction
// cache, and the weights of a thread's 8 channels arrive as 16-byte vectors when the weight
// tensor is contiguous [dim, W].  Small groups keep the registers low and the SMs full of
// CTAs: depth 2 measured fastest (depth 8 single-buffered was 10% slower).
constexpr int kPipeTile = 64;
constexpr int kPipeDepth = 2;

template <typename T, typename TW, int W>
__global__ void __launch_bounds__(128) conv1d_fwd_pipe_kernel(ConvParams p) {
  int seq, pos0;
  if (!find_tile(p.cu, p.n_seqs, kPipeTile, blockIdx.x, seq, pos0)) return;
  const int c0 = (blockIdx.y * 128 + threadIdx.x) * 8;
  if (c0 >= p.dim) return;
  const int start = p.cu[seq];
  const int L = p.cu[seq + 1] - start;
  const int pend = min(L, pos0 + kPipeTile);
  const T* x = static_cast<const T*>(p.x) + c0;
  T* st = static_cast<T*>(p.state) + (int64_t)p.idx[seq] * p.ss_n + c0;
  T* out = static_cast<T*>(p.out) + c0;

  float w[W][8];
  const TW* wp = static_cast<const TW*>(p.w) + (int64_t)c0 * p.sw_c;
  constexpr int kWv = 16 / sizeof(TW);  // weights per 16-byte vector
  if (p.sw_j == 1 && p.sw_c == W && (8 * W) % kWv == 0 && (reinterpret_cast<uintptr_t>(wp) & 15) == 0) {
    TW wl[8 * W];
#pragma unroll
    for (int v = 0; v < 8 * W / kWv; ++v) reinterpret_cast<uint4*>(wl)[v] = reinterpret_cast<const uint4*>(wp)[v];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int j = 0; j < W; ++j) w[j][i] = to_f32<TW>(wl[i * W + j]);
  } else {
#pragma unroll
    for (int j = 0; j < W; ++j)
#pragma unroll
      for (int i = 0; i < 8; ++i) w[j][i] = to_f32<TW>(wp[(int64_t)i * p.sw_c + j * p.sw_j]);
  }

  // window rows xp[pos0 + j], j < W-1 (xp index e < W-1 is state row e, else x[start + e - (W-1)])
  float win[W][8];
#pragma unroll
  for (int j = 0; j < W - 1; ++j) {
    const int e = pos0 + j;
    const T* src = e < W - 1 ? st + e * p.ss_t : x + (int64_t)(start + e - (W - 1)) * p.sx_t;
    unpack8<T>(*reinterpret_cast<const uint4*>(src), win[j]);
  }
  // new conv state: the tile holding position 0 is the only reader of the old state
  if (pos0 == 0) {
    uint4 ns[W - 1];
#pragma unroll
    for (int j = 0; j < W - 1; ++j) {
      const int e = L + j;
      ns[j] = *reinterpret_cast<const uint4*>(e < W - 1 ? st + e * p.ss_t : x + (int64_t)(start + e - (W - 1)) * p.sx_t);
    }
#pragma unroll
    for (int j = 0; j < W - 1; ++j) *reinterpret_cast<uint4*>(st + j * p.ss_t) = ns[j];
  }

  uint4 rows[kPipeDepth];
#pragma unroll
  for (int b = 0; b < kPipeDepth; ++b)
    if (pos0 + b < pend) rows[b] = __ldcs(reinterpret_cast<const uint4*>(x + (int64_t)(start + pos0 + b) * p.sx_t));
#pragma unroll 1
  for (int t0 = pos0; t0 < pend; t0 += kPipeDepth) {
    uint4 nxt[kPipeDepth];
#pragma unroll
    for (int b = 0; b < kPipeDepth; ++b)
      if (t0 + kPipeDepth + b < pend)
        nxt[b] = __ldcs(reinterpret_cast<const uint4*>(x + (int64_t)(start + t0 + kPipeDepth + b) * p.sx_t));
#pragma unroll
    for (int b = 0; b < kPipeDepth; ++b) {
      if (t0 + b < pend) {
        unpack8<T>(rows[b], win[W - 1]);
        float acc[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          float a = 0.f;
#pragma unroll
          for (int j = 0; j < W; ++j) a += w[j][i] * win[j][i];
          acc[i] = p.silu ? silu_fast(a) : a;
        }
        __stcs(reinterpret_cast<uint4*>(out + (int64_t)(start + t0 + b) * p.so_t), pack8<T>(acc));
#pragma unroll
        for (int j = 0; j < W - 1; ++j)
#pragma unroll
          for (int i = 0; i < 8; ++i) win[j][i] = win[j + 1][i];
      }
    }
#pragma unroll
    for (int b = 0; b < kPipeDepth; ++b) rows[b] = nxt[b];
  }
}

// Decode: one token per sequence; grid (dim / (128 VEC), S).
template <typename T, typename TW, int VEC, int W>
__global__ void __launch_bounds__(128) conv1d_update_kernel(ConvParams p) {
  const int seq = blockIdx.y;
  const int c0 = (blockIdx.x * blockDim.x + threadIdx.x) * VEC;
  if (c0 >= p.dim) return;
  const T* x = static_cast<const T*>(p.x) + (int64_t)seq * p.sx_t + c0 * p.sx_c;
  const TW* wp = static_cast<const TW*>(p.w);
  T* st = static_cast<T*>(p.state) + (int64_t)p.idx[seq] * p.ss_n + c0 * p.ss_c;
  T* out = static_cast<T*>(p.out) + (int64_t)seq * p.so_t + c0 * p.so_c;

  float xp[kMaxW][VEC];
#pragma unroll
  for (int j = 0; j < kMaxW - 1; ++j)
    if (j < W - 1) load_vec<T, TW, VEC>(st + j * p.ss_t, p.ss_c, xp[j]);
  float cur[VEC];
  load_vec<T, TW, VEC>(x, p.sx_c, cur);
  // weights: the thread's VEC x W taps as 16-byte vectors when [dim, W] is contiguous (one
  // scalar load per tap otherwise)
  float w[W][VEC];
  const TW* wt = wp + (int64_t)c0 * p.sw_c;
  constexpr int kWv = 16 / sizeof(TW);
  if (VEC == 8 && p.sw_j == 1 && p.sw_c == W && (VEC * W) % kWv == 0 && (reinterpret_cast<uintptr_t>(wt) & 15) == 0) {
    TW wl[VEC * W];
#pragma unroll
    for (int v = 0; v < VEC * W / kWv; ++v) reinterpret_cast<uint4*>(wl)[v] = reinterpret_cast<const uint4*>(wt)[v];
#pragma unroll
    for (int i = 0; i < VEC; ++i)
#pragma unroll
      for (int j = 0; j < W; ++j) w[j][i] = to_f32<TW>(wl[i * W + j]);
  } else {
#pragma unroll
    for (int j = 0; j < W; ++j)
#pragma unroll
      for (int i = 0; i < VEC; ++i) w[j][i] = to_f32<TW>(wt[(int64_t)i * p.sw_c + j * p.sw_j]);
  }
  float acc[VEC];
#pragma unroll
  for (int i = 0; i < VEC; ++i) {
    float a = 0.f;
#pragma unroll
    for (int j = 0; j < W; ++j) a += w[j][i] * (j == W - 1 ? cur[i] : xp[j][i]);
    acc[i] = p.silu ? silu_fast(a) : a;
  }
  store_vec<T, VEC>(out, p.so_c, acc);
#pragma unroll
  for (int j = 0; j < kMaxW - 1; ++j) {
    if (j < W - 1) {
      if (j + 1 < W - 1)
        store_vec<T, VEC>(st + j * p.ss_t, p.ss_c, xp[j + 1]);
      else
        store_vec<T, VEC>(st + j * p.ss_t, p.ss_c, cur);
    }
  }
}

template <typename T, typename TW, int W>
void launch_w(bool prefill, bool vec8, const ConvParams& p, int64_t T_tokens, cudaStream_t st) {
  const int VEC = vec8 ? 8 : 1;
  const int chan_blocks = (p.dim + 128 * VEC - 1) / (128 * VEC);
  if (prefill) {
    if (vec8) {
      dim3 grid((unsigned)((T_tokens + kPipeTile - 1) / kPipeTile + p.n_seqs), chan_blocks);
      conv1d_fwd_pipe_kernel<T, TW, W><<<grid, 128, 0, st>>>(p);
    } else {
      dim3 grid((unsigned)((T_tokens + p.tile - 1) / p.tile + p.n_seqs), chan_blocks);
      conv1d_fwd_kernel<T, TW, 1, W><<<grid, 128, 0, st>>>(p);
    }
  } else {
    dim3 grid(chan_blocks, p.n_seqs);
    if (vec8) conv1d_update_kernel<T, TW, 8, W><<<grid, 128, 0, st>>>(p);
    else conv1d_update_kernel<T, TW, 1, W><<<grid, 128, 0, st>>>(p);
  }
}

template <typename T, typename TW>
void launch(bool prefill, bool vec8, const ConvParams& p, int64_t T_tokens, cudaStream_t st) {
  switch (p.width) {
    case 2: launch_w<T, TW, 2>(prefill, vec8, p, T_tokens, st); break;
    case 3: launch_w<T, TW, 3>(prefill, vec8, p, T_tokens, st); break;
    case 4: launch_w<T, TW, 4>(prefill, vec8, p, T_tokens, st); break;
    case 5: launch_w<T, TW, 5>(prefill, vec8, p, T_tokens, st); break;
    case 6: launch_w<T, TW, 6>(prefill, vec8, p, T_tokens, st); break;
  }
}

int run_conv(const char* op, bool prefill, const mvb_tensor* x, const mvb_tensor* w, mvb_tensor* state,
             const mvb_tensor* idx, const mvb_tensor* cu, mvb_tensor* out, int activation, cudaStream_t st) {
  int rc;
  if ((rc = check_tensor(x, op, "x", 2)) || (rc = check_tensor(w, op, "weight", 2)) ||
      (rc = check_tensor(state, op, "conv_state", 3)) || (rc = check_tensor(idx, op, "conv_state_indices", 1)) ||
      (rc = check_tensor(out, op, "out", 2)))
    return rc;
  const int64_t T = x->shape[0], dim = x->shape[1], W = w->shape[1];
  MVB_CHECK_ARG(w->shape[0] == dim, "%s: weight must be [dim, W]", op);
  MVB_CHECK_SUPPORTED(W >= kMinW && W <= kMaxW, "%s: kernel width %lld not in [%d, %d]", op, (long long)W, kMinW,
                      kMaxW);
  MVB_CHECK_ARG(state->shape[1] == W - 1 && state->shape[2] == dim, "%s: conv_state must be [S_max, W-1, dim]", op);
  MVB_CHECK_ARG(out->shape[0] == T && out->shape[1] == dim, "%s: out must match x", op);
  MVB_CHECK_ARG(x->dtype == out->dtype && x->dtype == state->dtype && is_float_dtype(x->dtype),
                "%s: x, conv_state and out must share one float dtype", op);
  MVB_CHECK_ARG(w->dtype == MVB_F32 || w->dtype == x->dtype, "%s: weight must be float32 or x's dtype", op);
  MVB_CHECK_ARG(idx->dtype == MVB_I32, "%s: conv_state_indices must be int32", op);
  int64_t n_seqs = T;
  if (prefill) {
    if ((rc = check_tensor(cu, op, "cu_seqlens", 1))) return rc;
    MVB_CHECK_ARG(cu->dtype == MVB_I32 && cu->shape[0] >= 1, "%s: cu_seqlens must be int32 [S+1]", op);
    n_seqs = cu->shape[0] - 1;
  }
  MVB_CHECK_ARG(idx->shape[0] >= n_seqs, "%s: conv_state_indices shorter than the batch", op);
  MVB_CHECK_SUPPORTED(n_seqs <= 65535 || prefill, "%s: at most 65535 sequences per launch", op);
  if (n_seqs == 0 || dim == 0) return MVB_OK;

  ConvParams p;
  p.x = x->data; p.w = w->data; p.state = state->data; p.idx = static_cast<const int32_t*>(idx->data);
  p.cu = prefill ? static_cast<const int32_t*>(cu->data) : nullptr; p.out = out->data;
  p.sx_t = x->stride[0]; p.sx_c = x->stride[1]; p.sw_c = w->stride[0]; p.sw_j = w->stride[1];
  p.ss_n = state->stride[0]; p.ss_t = state->stride[1]; p.ss_c = state->stride[2];
  p.so_t = out->stride[0]; p.so_c = out->stride[1];
  p.n_seqs = (int)n_seqs; p.dim = (int)dim; p.width = (int)W; p.silu = activation ? 1 : 0; p.tile = 64;

  const int es = dtype_size(x->dtype);
  const bool vec8 = es == 2 && dim % 8 == 0 && p.sx_c == 1 && p.ss_c == 1 && p.so_c == 1 && aligned16(p.x) &&
                    aligned16(p.state) && aligned16(p.out) && (p.sx_t * es) % 16 == 0 &&
                    (p.ss_t * es) % 16 == 0 && (p.ss_n * es) % 16 == 0 && (p.so_t * es) % 16 == 0;
  const bool w32 = w->dtype == MVB_F32;
  switch (x->dtype) {
    case MVB_F32: launch<float, float>(prefill, false, p, T, st); break;
    case MVB_BF16:
      if (w32) launch<__nv_bfloat16, float>(prefill, vec8, p, T, st);
      else launch<__nv_bfloat16, __nv_bfloat16>(prefill, vec8, p, T, st);
      break;
    case MVB_F16:
      if (w32) launch<__half, float>(prefill, vec8, p, T, st);
      else launch<__half, __half>(prefill, vec8, p, T, st);
      break;
  }
  MVB_CHECK_LAUNCH(op);
  return MVB_OK;
}

}  // namespace
}  // namespace mvb

extern "C" int mvb_causal_conv1d_fn(const mvb_tensor* x, const mvb_tensor* weight, mvb_tensor* conv_state,
                                    const mvb_tensor* conv_state_indices, const mvb_tensor* cu_seqlens,
                                    mvb_tensor* out, int activation, void* stream) {
  return mvb::run_conv("causal_conv1d_fn", true, x, weight, conv_state, conv_state_indices, cu_seqlens, out,
                       activation, static_cast<cudaStream_t>(stream));
}

extern "C" int mvb_causal_conv1d_update(const mvb_tensor* x, const mvb_tensor* weight, mvb_tensor* conv_state,
                                        const mvb_tensor* conv_state_indices, mvb_tensor* out, int activation,
                                        void* stream) {
  return mvb::run_conv("causal_conv1d_update", false, x, weight, conv_state, conv_state_indices, nullptr, out,
                       activation, static_cast<cudaStream_t>(stream));
}
