// Paged-KV decode attention (one query per sequence), HBM-bound.
//
// Replaces _paged_flash_attention_decode_kernel (m/ops/full_attention.py:176-279), which
// runs one program per (seq, q-head) and so streams every KV page once per q-head
// (8x for GQA 8:1).  Here one CTA owns (split, kv-head, seq) and computes all G =
// Hq / Hkv query heads of that kv-head together, so each cached K/V row crosses HBM
// once:
//   S[g, t] = scale q_g . k_t ;  online softmax over t (exp2, fp32) ;  O[g] = sum p v_t
// Tiles of 64 tokens are gathered through the block table (the split's entries are first
// copied to shared memory) with 16-byte cp.async into an XOR-swizzled NSTAGE-deep
// shared-memory ring, so NSTAGE-1 tiles are in flight while one is computed; when the
// block size is a multiple of 64 a tile lies in one page.  Each of the 4 warps takes 16
// tokens of a tile and runs QK^T and PV on mma.sync m16n8k16 (G padded to 16 rows;
// the padded rows are never written).  Long contexts are split across CTAs
// (flash-decoding); split results (normalised O and log2-sum-exp) go to the caller's
// workspace and a second kernel merges them.  With long splits, a one-block kernel first
// orders the split work largest first (every full split, then the partial last splits by
// length), so that the last wave of CTAs holds the shortest items instead of whatever the
// grid order left there.
#include <mutex>

#include "common.cuh"

namespace mvb {

struct DecodeParams {
  const void* q;
  const void *kc, *vc;
  const int32_t* bt;
  const int32_t* ctx;
  void* o;
  const void* gate;  // [S, Hq, Dv] output gate (o *= sigmoid(gate)), or null
  int64_t sgt_s, sgt_h;
  float* part_o;     // [S, Hkv, n_splits, 16, Dv] fp32, or null when n_splits == 1
  float* part_lse;   // [S, Hkv, n_splits, 16]
  // Context parts (a kv head's context shared out among n_parts ranks): this call runs the
  // splits s with s % n_parts == part and leaves their merge, normalised within the part, in
  // o_part [S, Hq, Dv] fp32 with its log2-sum-exp in lse_part [S, Hq].  n_parts == 1: off.
  int part, n_parts;
  float *o_part, *lse_part;
  // Largest-first order of the split work (null: grid order), int32 [2 S + 2]: [0, S] the
  // prefix sums of each sequence's full splits run by this call; [S + 1, S + 1 + n) the n
  // sequences whose partial last split this call runs, longest first; [2 S + 1] n.
  const int* order;
  int n_seqs;
  int64_t sq_s, sq_h, so_s, so_h;
  int64_t skc_b, skc_t, skc_h, svc_b, svc_t, svc_h;
  int64_t sbt_s, sbt_b;
  int hq, hkv, group, block_size, max_blocks, n_splits, split_len;
  float scale_log2;  // scale * log2(e)
};

namespace {

constexpr int kTile = 64;
constexpr int kWarps = 4;

constexpr int kMaxSplitPages = 1024;  // block-table entries of one split cached in smem
constexpr int kMaxOrderedSeqs = 4096;  // larger batches run their splits in grid order

template <int D>
struct DecodeSmem {
  static constexpr int kStages = D >= 256 ? 3 : 4;
  static constexpr int kRowBytes = D * 2;
  static constexpr int kTileBytes = kTile * kRowBytes;
  static constexpr int kStageBytes = 2 * kTileBytes;  // K + V
  static constexpr int kQBytes = 16 * kRowBytes;
  static constexpr int kPagesBytes = kMaxSplitPages * 4;
  static constexpr int kBytes = kStages * kStageBytes + kQBytes + kPagesBytes;
};

// Byte offset of 16-byte chunk `c` of row `r` in a swizzled [rows][D] bf16 tile.
template <int D>
__device__ __forceinline__ int swz(int r, int c) {
  return r * (D * 2) + ((c ^ (r & 7)) << 4);
}

// sigmoid(gate[seq, head, c]) of the gated-attention output (fp32 math, one rounding of the
// product instead of torch's rounding of the sigmoid and of the product).
template <typename T>
__device__ __forceinline__ float sigmoid_gate(const DecodeParams& p, int seq, int head, int c) {
  const float g = to_f32<T>(static_cast<const T*>(p.gate)[(int64_t)seq * p.sgt_s + (int64_t)head * p.sgt_h + c]);
  return 1.f / (1.f + __expf(-g));
}

// Block-table entry for token t: from the split's smem copy when it holds it.
__device__ __forceinline__ int page_of(const DecodeParams& p, const int* spages, int page0, int npages, int seq,
                                       int t) {
  const int pg = t / p.block_size;
  return (pg - page0 < npages) ? spages[pg - page0] : p.bt[seq * p.sbt_s + pg * p.sbt_b];
}

template <typename T, int D>
__device__ __forceinline__ void load_tile(const DecodeParams& p, char* sK, char* sV, const int* spages, int page0,
                                          int npages, int seq, int kvh, int t0, int ctx) {
  constexpr int CH = D / 8;  // 16-byte chunks per row
  const char* kc = static_cast<const char*>(p.kc);
  const char* vc = static_cast<const char*>(p.vc);
  if (p.block_size % kTile == 0) {  // the whole tile lies in one page
    const int64_t blk = page_of(p, spages, page0, npages, seq, t0);
    const int off0 = t0 % p.block_size;
    const char* kb = kc + (blk * p.skc_b + kvh * p.skc_h) * 2;
    const char* vb = vc + (blk * p.svc_b + kvh * p.svc_h) * 2;
    for (int i = threadIdx.x; i < kTile * CH; i += kWarps * 32) {
      const int r = i / CH, c = i % CH;
      const bool ok = t0 + r < ctx;
      const int64_t row = ok ? off0 + r : 0;
      cp_async16(sK + swz<D>(r, c), kb + row * p.skc_t * 2 + c * 16, ok);
      cp_async16(sV + swz<D>(r, c), vb + row * p.svc_t * 2 + c * 16, ok);
    }
    return;
  }
  for (int i = threadIdx.x; i < kTile * CH; i += kWarps * 32) {
    const int r = i / CH, c = i % CH;
    const int t = t0 + r;
    const bool ok = t < ctx;
    int64_t koff = 0, voff = 0;
    if (ok) {
      const int64_t blk = page_of(p, spages, page0, npages, seq, t);
      const int off = t % p.block_size;
      koff = (blk * p.skc_b + off * p.skc_t + kvh * p.skc_h) * 2 + c * 16;
      voff = (blk * p.svc_b + off * p.svc_t + kvh * p.svc_h) * 2 + c * 16;
    }
    cp_async16(sK + swz<D>(r, c), kc + koff, ok);
    cp_async16(sV + swz<D>(r, c), vc + voff, ok);
  }
}

// Item i of the largest-first order -> (seq, split); false past the last item.  Items are
// every sequence's full splits (prefix sums in order[0..S]), then the partial last splits
// longest first (sequence ids in order[S+1..]).
__device__ __forceinline__ bool ordered_item(const DecodeParams& p, int i, int& seq, int& split) {
  const int S = p.n_seqs;
  const int n_full = p.order[S];
  if (i < n_full) {
    int lo = 0, hi = S - 1;  // the last s with order[s] <= i
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (p.order[mid] <= i) lo = mid;
      else hi = mid - 1;
    }
    seq = lo;
    split = p.part + (i - p.order[lo]) * p.n_parts;
    return true;
  }
  const int k = i - n_full;
  if (k >= p.order[2 * S + 1]) return false;
  seq = p.order[S + 1 + k];
  split = min(p.ctx[seq], p.n_splits * p.split_len) / p.split_len;
  return true;
}

// One block: the largest-first order of a decode call's split work (see DecodeParams).
// Split j of sequence s is full when (j + 1) L <= ctx_s and partial when j L < ctx_s <
// (j + 1) L; this call runs the splits with j % n_parts == part.
__global__ void __launch_bounds__(256) decode_order_kernel(DecodeParams p, int* order) {
  __shared__ int s_warp[32];
  __shared__ int s_np;
  __shared__ int s_key[kMaxOrderedSeqs];
  const int S = p.n_seqs, L = p.split_len, tid = threadIdx.x;
  // full splits of this part, per sequence, and an exclusive prefix sum over them
  int carry = 0;
  for (int base = 0; base < S; base += blockDim.x) {
    const int s = base + tid;
    int f = 0;
    if (s < S) {
      const int fa = min(p.ctx[s], p.n_splits * L) / L;  // (a context never exceeds the bound)
      f = fa > p.part ? (fa - p.part + p.n_parts - 1) / p.n_parts : 0;
    }
    int x = f;  // inclusive scan over the block
    const int lane = tid & 31, w = tid >> 5;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) s_warp[w] = x;
    __syncthreads();
    if (w == 0) {
      int v = lane < (int)(blockDim.x >> 5) ? s_warp[lane] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += y;
      }
      s_warp[lane] = v;
    }
    __syncthreads();
    const int incl = x + (w > 0 ? s_warp[w - 1] : 0) + carry;
    if (s < S) order[s] = incl - f;
    carry += s_warp[(blockDim.x >> 5) - 1];
    __syncthreads();
  }
  if (tid == 0) {
    order[S] = carry;
    s_np = 0;
  }
  // partial last splits run by this part, ranked longest first (ties: lower sequence first);
  // keys in shared memory (the partial's length, -1 where this part runs none)
  for (int s = tid; s < S; s += blockDim.x) {
    const int c = min(p.ctx[s], p.n_splits * L), r = c % L, j = c / L;
    s_key[s] = (r == 0 || j % p.n_parts != p.part) ? -1 : r;
  }
  __syncthreads();
  int np = 0;
  for (int s = tid; s < S; s += blockDim.x) {
    const int r = s_key[s];
    if (r < 0) continue;
    int rank = 0;
    for (int t = 0; t < S; ++t) {
      const int rt = s_key[t];
      rank += (rt > r) || (rt == r && t < s);
    }
    order[S + 1 + rank] = s;
    ++np;
  }
  if (np > 0) atomicAdd(&s_np, np);
  __syncthreads();
  if (tid == 0) order[2 * S + 1] = s_np;
}

template <typename T, int D>
__global__ void __launch_bounds__(kWarps * 32) paged_decode_kernel(DecodeParams p) {
  using SM = DecodeSmem<D>;
  constexpr int NS = SM::kStages;
  extern __shared__ __align__(128) char smem[];
  char* sQ = smem + NS * SM::kStageBytes;
  int* spages = reinterpret_cast<int*>(sQ + SM::kQBytes);
  int split, kvh, seq;
  if (p.order == nullptr) {
    split = blockIdx.x * p.n_parts + p.part, kvh = blockIdx.y, seq = blockIdx.z;
  } else if (!ordered_item(p, blockIdx.y, seq, split)) {
    return;  // past the last item: no work (the merge skips splits past a context)
  } else {
    kvh = blockIdx.x;
  }
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int ctx = p.ctx[seq];
  const int t_begin = split * p.split_len;
  const int t_end = min(ctx, t_begin + p.split_len);
  const int G = p.group;

  if (t_begin >= t_end) {
    if (p.part_o != nullptr && tid < 16) {
      const int64_t pi = ((int64_t)seq * p.hkv + kvh) * p.n_splits + split;
      p.part_lse[pi * 16 + tid] = -INFINITY;
    } else if (p.part_o == nullptr) {  // empty context: zeros
      T* o = static_cast<T*>(p.o);
      for (int i = tid; i < G * D; i += kWarps * 32)
        o[seq * p.so_s + (kvh * G + i / D) * p.so_h + i % D] = from_f32<T>(0.f);
    }
    return;
  }

  // Q -> smem (rows >= G zero).
  {
    const T* q = static_cast<const T*>(p.q);
    constexpr int CH = D / 8;
    for (int i = tid; i < 16 * CH; i += kWarps * 32) {
      const int r = i / CH, c = i % CH;
      uint4 val = make_uint4(0, 0, 0, 0);
      if (r < G) val = *reinterpret_cast<const uint4*>(q + seq * p.sq_s + (kvh * G + r) * p.sq_h + c * 8);
      *reinterpret_cast<uint4*>(sQ + swz<D>(r, c)) = val;
    }
  }

  // this split's block-table entries -> smem
  const int page0 = t_begin / p.block_size;
  const int npages = min((t_end - 1) / p.block_size - page0 + 1, kMaxSplitPages);
  for (int i = tid; i < npages; i += kWarps * 32) spages[i] = p.bt[seq * p.sbt_s + (page0 + i) * p.sbt_b];
  __syncthreads();

  const int n_tiles = (t_end - t_begin + kTile - 1) / kTile;
#pragma unroll
  for (int st = 0; st < NS - 1; ++st) {
    if (st < n_tiles) {
      char* b = smem + st * SM::kStageBytes;
      load_tile<T, D>(p, b, b + SM::kTileBytes, spages, page0, npages, seq, kvh, t_begin + st * kTile, t_end);
    }
    cp_async_commit();
  }

  float acc[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;  // rows lane/4 and lane/4 + 8

  for (int it = 0; it < n_tiles; ++it) {
    const int stage = it % NS;
    cp_async_wait<NS - 2>();  // tile `it` has landed
    __syncthreads();          // ... for every thread, and stage (it - 1) % NS is free again
    if (it + NS - 1 < n_tiles) {
      char* nb = smem + ((it + NS - 1) % NS) * SM::kStageBytes;
      load_tile<T, D>(p, nb, nb + SM::kTileBytes, spages, page0, npages, seq, kvh, t_begin + (it + NS - 1) * kTile,
                      t_end);
    }
    cp_async_commit();
    const char* sK = smem + stage * SM::kStageBytes;
    const char* sV = sK + SM::kTileBytes;

    // S = Q K^T for this warp's 16 tokens (two n8 fragments).
    float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      uint32_t a[4], b[4];
      {
        const int r = lane & 15, c = kk * 2 + (lane >> 4);
        ldmatrix_x4(a[0], a[1], a[2], a[3], smem_u32(sQ + swz<D>(r, c)));
      }
      {
        // matrices: (tokens 0-7, k lo), (tokens 0-7, k hi), (tokens 8-15, k lo), (tokens 8-15, k hi)
        const int r = warp * 16 + (lane & 7) + ((lane >> 4) << 3);
        const int c = kk * 2 + ((lane >> 3) & 1);
        ldmatrix_x4(b[0], b[1], b[2], b[3], smem_u32(sK + swz<D>(r, c)));
      }
      mma16816<T>(s[0], a, b);
      mma16816<T>(s[1], a, b + 2);
    }
    // mask tokens past the end, scale into log2 domain
    const int tbase = t_begin + it * kTile + warp * 16 + (lane & 3) * 2;
#pragma unroll
    for (int n = 0; n < 2; ++n)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int t = tbase + n * 8 + (j & 1);
        s[n][j] = t < t_end ? s[n][j] * p.scale_log2 : -INFINITY;
      }
    float mx0 = fmaxf(fmaxf(s[0][0], s[0][1]), fmaxf(s[1][0], s[1][1]));
    float mx1 = fmaxf(fmaxf(s[0][2], s[0][3]), fmaxf(s[1][2], s[1][3]));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float nm0 = fmaxf(m0, mx0), nm1 = fmaxf(m1, mx1);
    // a warp whose 16 tokens are all masked keeps m = -inf: guard the rescale
    const float a0 = nm0 == -INFINITY ? 1.f : exp2f(m0 - nm0);
    const float a1 = nm1 == -INFINITY ? 1.f : exp2f(m1 - nm1);
    float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
    for (int n = 0; n < 2; ++n) {
      s[n][0] = nm0 == -INFINITY ? 0.f : exp2f(s[n][0] - nm0);
      s[n][1] = nm0 == -INFINITY ? 0.f : exp2f(s[n][1] - nm0);
      s[n][2] = nm1 == -INFINITY ? 0.f : exp2f(s[n][2] - nm1);
      s[n][3] = nm1 == -INFINITY ? 0.f : exp2f(s[n][3] - nm1);
      ps0 += s[n][0] + s[n][1];
      ps1 += s[n][2] + s[n][3];
    }
    l0 = l0 * a0 + ps0;
    l1 = l1 * a1 + ps1;
    m0 = nm0;
    m1 = nm1;
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
      acc[i][0] *= a0; acc[i][1] *= a0; acc[i][2] *= a1; acc[i][3] *= a1;
    }
    // P as the A operand (16 x 16 tokens) of PV.
    uint32_t pa[4];
    pa[0] = pack2<T>(s[0][0], s[0][1]);
    pa[1] = pack2<T>(s[0][2], s[0][3]);
    pa[2] = pack2<T>(s[1][0], s[1][1]);
    pa[3] = pack2<T>(s[1][2], s[1][3]);
#pragma unroll
    for (int nn = 0; nn < D / 16; ++nn) {
      uint32_t b[4];
      // V rows = tokens (k), 16 columns (two n8 fragments), transposed load.
      const int r = warp * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
      const int c = nn * 2 + (lane >> 4);
      ldmatrix_x4_trans(b[0], b[1], b[2], b[3], smem_u32(sV + swz<D>(r, c)));
      mma16816<T>(acc[nn * 2], pa, b);
      mma16816<T>(acc[nn * 2 + 1], pa, b + 2);
    }
  }
  cp_async_wait<0>();
  __syncthreads();  // the ring is reused for the cross-warp merge below

  // Row sums across the 4 lanes of a quad.
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);

  // Merge the 4 warps through shared memory (reuses the K/V ring).
  float* red = reinterpret_cast<float*>(smem);  // [4][16][D]
  float* sm = red + kWarps * 16 * D;            // [4][16] m
  float* sl = sm + kWarps * 16;                 // [4][16] l
  const int r0 = lane >> 2, r1 = r0 + 8;
  if ((lane & 3) == 0) {
    sm[warp * 16 + r0] = m0; sm[warp * 16 + r1] = m1;
    sl[warp * 16 + r0] = l0; sl[warp * 16 + r1] = l1;
  }
#pragma unroll
  for (int i = 0; i < D / 8; ++i) {
    const int c = i * 8 + (lane & 3) * 2;
    red[(warp * 16 + r0) * D + c] = acc[i][0];
    red[(warp * 16 + r0) * D + c + 1] = acc[i][1];
    red[(warp * 16 + r1) * D + c] = acc[i][2];
    red[(warp * 16 + r1) * D + c + 1] = acc[i][3];
  }
  __syncthreads();
  for (int i = tid; i < G * D; i += kWarps * 32) {
    const int r = i / D, c = i % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, sm[w * 16 + r]);
    float L = 0.f, O = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const float mw = sm[w * 16 + r];
      const float f = mw == -INFINITY ? 0.f : exp2f(mw - M);
      L += f * sl[w * 16 + r];
      O += f * red[(w * 16 + r) * D + c];
    }
    const float out = L > 0.f ? O / L : 0.f;
    if (p.part_o == nullptr) {
      T* o = static_cast<T*>(p.o);
      const float gt = p.gate ? sigmoid_gate<T>(p, seq, kvh * G + r, c) : 1.f;
      o[seq * p.so_s + (kvh * G + r) * p.so_h + c] = from_f32<T>(out * gt);
    } else {
      const int64_t pi = ((int64_t)seq * p.hkv + kvh) * p.n_splits + split;
      p.part_o[(pi * 16 + r) * D + c] = out;
      if (c == 0) p.part_lse[pi * 16 + r] = L > 0.f ? M + log2f(L) : -INFINITY;
    }
  }
}

// Merge split results: one CTA per (seq, q-head).
template <typename T, int D>
__global__ void __launch_bounds__(128) paged_decode_merge_kernel(DecodeParams p) {
  const int seq = blockIdx.y, hq = blockIdx.x;
  const int kvh = hq / p.group, r = hq % p.group;
  const int64_t base = ((int64_t)seq * p.hkv + kvh) * p.n_splits;
  // the splits this call ran: s = part + i n_parts (all of them, in order, without parts)
  const int n_own = p.part < p.n_splits ? (p.n_splits - p.part + p.n_parts - 1) / p.n_parts : 0;
  __shared__ float s_w[1024];
  __shared__ float s_tot;
  // splits that start past the context hold no keys (and, in largest-first order, no
  // partial was written for them)
  const int ctx = p.ctx[seq];
  auto lse_of = [&](int i) {
    const int sp = p.part + i * p.n_parts;
    return sp * p.split_len < ctx ? p.part_lse[(base + sp) * 16 + r] : -INFINITY;
  };
  float M = -INFINITY;
#pragma unroll 8
  for (int i = 0; i < n_own; ++i) M = fmaxf(M, lse_of(i));
  float tot = 0.f;
  for (int i = threadIdx.x; i < n_own; i += blockDim.x) {
    const float l = lse_of(i);
    const float w = l == -INFINITY ? 0.f : exp2f(l - M);
    s_w[i] = w;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int i = 0; i < n_own; ++i) tot += s_w[i];
    s_tot = tot;
  }
  __syncthreads();
  tot = s_tot;
  T* o = static_cast<T*>(p.o);
  for (int c = threadIdx.x; c < D; c += blockDim.x) {
    float acc = 0.f;
    // eight splits' loads in flight before their adds (a split past the context has weight
    // 0 and unwritten partials: the select keeps them out)
    for (int i0 = 0; i0 < n_own; i0 += 8) {
      float v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j)
        v[j] = i0 + j < n_own ? p.part_o[((base + p.part + (i0 + j) * p.n_parts) * 16 + r) * D + c] : 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (i0 + j < n_own && s_w[i0 + j] != 0.f) acc += s_w[i0 + j] * v[j];
    }
    const float out = tot > 0.f ? acc / tot : 0.f;
    if (p.o_part != nullptr) {  // this part's share, normalised within the part
      const int64_t oi = (int64_t)seq * p.hq + hq;
      p.o_part[oi * D + c] = out;
      if (c == 0) p.lse_part[oi] = tot > 0.f ? M + log2f(tot) : -INFINITY;
    } else {
      const float gt = p.gate ? sigmoid_gate<T>(p, seq, hq, c) : 1.f;
      o[seq * p.so_s + hq * p.so_h + c] = from_f32<T>(out * gt);
    }
  }
}

// The parts of a context split merged: o = o_part w (sigmoid(gate)), w = 2^(lse_own - M) /
// sum_j 2^(lse_j - M) over the parts j, M their max.  Summed over the parts, these outputs
// are the attention over the whole context; each part's output goes through the output
// projection on its own rank and the all-reduce after it adds them.  One CTA per (seq, q-head).
template <typename T, int D>
__global__ void __launch_bounds__(128) attention_parts_merge_kernel(const float* o_part, const float* lse_parts,
                                                                    int64_t sl_part, int n_parts, int part,
                                                                    const T* gate, int64_t sg_s, int64_t sg_h, T* o,
                                                                    int64_t so_s, int64_t so_h, int hq) {
  const int seq = blockIdx.y, h = blockIdx.x;
  const int64_t oi = (int64_t)seq * hq + h;
  float M = -INFINITY;
  for (int j = 0; j < n_parts; ++j) M = fmaxf(M, lse_parts[j * sl_part + oi]);
  float L = 0.f;
  for (int j = 0; j < n_parts; ++j) {
    const float l = lse_parts[j * sl_part + oi];
    L += l == -INFINITY ? 0.f : exp2f(l - M);
  }
  const float own = lse_parts[part * sl_part + oi];
  const float w = (L > 0.f && own != -INFINITY) ? exp2f(own - M) / L : 0.f;
  for (int c = threadIdx.x; c < D; c += blockDim.x) {
    float g = 1.f;
    if (gate != nullptr) g = 1.f / (1.f + __expf(-to_f32<T>(gate[seq * sg_s + h * sg_h + c])));
    o[seq * so_s + h * so_h + c] = from_f32<T>(w == 0.f ? 0.f : o_part[oi * D + c] * w * g);
  }
}

}  // namespace

constexpr int kMaxSplits = 1024;

// Chooses the split length (a multiple of the tile) for a context bound and batch.
// With a context split over n_parts ranks each rank runs 1 / n_parts of the splits, so
// there are n_parts times as many.
inline int decode_split_len(int64_t n_seqs, int64_t hkv, int64_t max_ctx, int64_t max_splits, int64_t n_parts = 1) {
  if (max_splits <= 1) return (int)(((max_ctx + kTile - 1) / kTile) * kTile);  // one split: the whole context
  const int64_t per = n_seqs * hkv;
  // aim for >= 8 CTAs per SM of work (16 measured the same at config 4; 32 and more were
  // 45% slower)
  int64_t target = (8LL * 148 * n_parts + per - 1) / (per > 0 ? per : 1);
  int64_t split = (max_ctx + target - 1) / (target > 0 ? target : 1);
  split = ((split + kTile - 1) / kTile) * kTile;
  if (split < 512) split = 512;
  while ((max_ctx + split - 1) / split > max_splits) split += kTile;
  return (int)split;
}

size_t decode_workspace_bytes(int64_t n_seqs, int64_t hkv, int64_t dv, int n_splits, bool parts = false) {
  if (n_splits <= 1 && !parts) return 0;
  return (size_t)n_seqs * hkv * n_splits * 16 * (dv + 1) * sizeof(float);
}

// The largest-first order table after the split partials (int32 [2 S + 2], 16-byte padded).
// A call whose workspace lacks this room runs the splits in grid order.
size_t decode_order_bytes(int64_t n_seqs) { return (size_t)((2 * n_seqs + 2) * 4 + 15) / 16 * 16; }
size_t decode_workspace_bytes_ordered(int64_t n_seqs, int64_t hkv, int64_t dv, int n_splits, bool parts = false) {
  const size_t b = decode_workspace_bytes(n_seqs, hkv, dv, n_splits, parts);
  return b == 0 || n_seqs > kMaxOrderedSeqs ? b : b + decode_order_bytes(n_seqs);
}

namespace {
// Internal linkage on purpose: a function-local static of a template with external linkage
// is a unique symbol that the dynamic loader merges across every loaded copy of the
// library, so a second copy would skip setting the shared-memory attribute of its own kernel.
template <typename T, int D>
int launch_decode(DecodeParams& p, int64_t n_seqs, cudaStream_t st) {
  const int smem = DecodeSmem<D>::kBytes;
  static unsigned long long attr_mask = 0;
  ensure_smem_attr(paged_decode_kernel<T, D>, smem, attr_mask);
  const int n_own = p.part < p.n_splits ? (p.n_splits - p.part + p.n_parts - 1) / p.n_parts : 0;
  if (n_own > 0 && p.order != nullptr) {  // largest-first: (kv head, item), items ordered on device
    decode_order_kernel<<<1, 256, 0, st>>>(p, const_cast<int*>(p.order));
    dim3 grid(p.hkv, (unsigned)(n_seqs * n_own));
    paged_decode_kernel<T, D><<<grid, kWarps * 32, smem, st>>>(p);
  } else if (n_own > 0) {
    dim3 grid(n_own, p.hkv, (unsigned)n_seqs);
    paged_decode_kernel<T, D><<<grid, kWarps * 32, smem, st>>>(p);
  }
  if (p.part_o != nullptr) {
    dim3 g2(p.hq, (unsigned)n_seqs);
    paged_decode_merge_kernel<T, D><<<g2, 128, 0, st>>>(p);
  }
  return MVB_OK;
}
}  // namespace

// Shared by the workspace and the static-scratch entry points.
int run_paged_decode(const char* op, const mvb_tensor* q, const mvb_tensor* kc, const mvb_tensor* vc,
                     const mvb_tensor* bt, const mvb_tensor* ctx, float scale, int block_size, int64_t max_ctx,
                     mvb_tensor* o, void* ws, size_t ws_bytes, int64_t max_splits, cudaStream_t st,
                     const mvb_tensor* gate = nullptr, int part = 0, int n_parts = 1,
                     mvb_tensor* lse_part = nullptr) {
  // lse_part set: a context part (o is then the part's fp32 output [S, Hq, Dv], contiguous)
  const bool parts = lse_part != nullptr;
  int rc;
  if ((rc = check_tensor(q, op, "q", 3)) || (rc = check_tensor(kc, op, "k_cache", 4)) ||
      (rc = check_tensor(vc, op, "v_cache", 4)) || (rc = check_tensor(bt, op, "block_tables", 2)) ||
      (rc = check_tensor(ctx, op, "context_lens", 1)) || (rc = check_tensor(o, op, "o", 3)))
    return rc;
  const int64_t S = q->shape[0], hq = q->shape[1], d = q->shape[2];
  const int64_t hkv = kc->shape[2], dv = vc->shape[3];
  MVB_CHECK_ARG(kc->shape[1] == block_size && vc->shape[1] == block_size && block_size > 0,
                "%s: caches must be [n_blocks, block_size=%d, Hkv, D]", op, block_size);
  MVB_CHECK_ARG(kc->shape[3] == d && vc->shape[2] == hkv && vc->shape[0] == kc->shape[0],
                "%s: k_cache/v_cache shapes disagree with q", op);
  MVB_CHECK_ARG(hkv > 0 && hq % hkv == 0, "%s: Hq must be a multiple of Hkv", op);
  MVB_CHECK_ARG(o->shape[0] == S && o->shape[1] == hq && o->shape[2] == dv, "%s: o must be [S, Hq, Dv]", op);
  MVB_CHECK_ARG(bt->shape[0] >= S && ctx->shape[0] >= S && bt->dtype == MVB_I32 && ctx->dtype == MVB_I32,
                "%s: block_tables [S, max_blocks] and context_lens [S] must be int32", op);
  MVB_CHECK_ARG(q->dtype == kc->dtype && q->dtype == vc->dtype && (parts ? o->dtype == MVB_F32 : q->dtype == o->dtype),
                "%s: dtype mismatch", op);
  if (parts) {
    if ((rc = check_tensor(lse_part, op, "lse_part", 2))) return rc;
    MVB_CHECK_ARG(n_parts >= 1 && part >= 0 && part < n_parts, "%s: part %d of %d", op, part, n_parts);
    MVB_CHECK_ARG(lse_part->shape[0] == S && lse_part->shape[1] == hq && lse_part->dtype == MVB_F32,
                  "%s: lse_part must be [S, Hq] fp32", op);
    MVB_CHECK_SUPPORTED(o->stride[0] == hq * dv && o->stride[1] == dv && lse_part->stride[0] == hq &&
                            lse_part->stride[1] == 1,
                        "%s: o_part and lse_part must be contiguous", op);
  }
  MVB_CHECK_SUPPORTED(q->dtype == MVB_BF16 || q->dtype == MVB_F16, "%s: q/k/v must be bf16 or fp16", op);
  MVB_CHECK_SUPPORTED(d == dv && (d == 64 || d == 128 || d == 256), "%s: head dim must be 64, 128 or 256", op);
  MVB_CHECK_SUPPORTED(hq / hkv <= 16, "%s: at most 16 query heads per kv head", op);
  MVB_CHECK_SUPPORTED(q->stride[2] == 1 && o->stride[2] == 1 && kc->stride[3] == 1 && vc->stride[3] == 1 &&
                          q->stride[1] % 8 == 0 && q->stride[0] % 8 == 0 && kc->stride[0] % 8 == 0 &&
                          kc->stride[1] % 8 == 0 && kc->stride[2] % 8 == 0 && vc->stride[0] % 8 == 0 &&
                          vc->stride[1] % 8 == 0 && vc->stride[2] % 8 == 0 && aligned16(q->data) &&
                          aligned16(kc->data) && aligned16(vc->data),
                      "%s: rows must be contiguous and 16-byte aligned", op);
  MVB_CHECK_SUPPORTED(S <= 65535 && hkv <= 65535, "%s: too many sequences", op);
  if (S == 0 || hq == 0) return MVB_OK;
  if (max_ctx <= 0) max_ctx = bt->shape[1] * (int64_t)block_size;
  if (max_ctx <= 0) max_ctx = 1;

  DecodeParams p;
  p.q = q->data; p.kc = kc->data; p.vc = vc->data;
  p.bt = static_cast<const int32_t*>(bt->data); p.ctx = static_cast<const int32_t*>(ctx->data); p.o = o->data;
  p.gate = nullptr; p.sgt_s = p.sgt_h = 0;
  if (gate != nullptr) {
    if ((rc = check_tensor(gate, op, "gate", 3))) return rc;
    MVB_CHECK_ARG(gate->shape[0] == S && gate->shape[1] == hq && gate->shape[2] == dv && gate->dtype == q->dtype,
                  "%s: gate must be [S, Hq, Dv] in the dtype of q", op);
    MVB_CHECK_SUPPORTED(gate->stride[2] == 1, "%s: gate needs a unit last stride", op);
    p.gate = gate->data; p.sgt_s = gate->stride[0]; p.sgt_h = gate->stride[1];
  }
  p.sq_s = q->stride[0]; p.sq_h = q->stride[1]; p.so_s = o->stride[0]; p.so_h = o->stride[1];
  p.skc_b = kc->stride[0]; p.skc_t = kc->stride[1]; p.skc_h = kc->stride[2];
  p.svc_b = vc->stride[0]; p.svc_t = vc->stride[1]; p.svc_h = vc->stride[2];
  p.sbt_s = bt->stride[0]; p.sbt_b = bt->stride[1];
  p.hq = (int)hq; p.hkv = (int)hkv; p.group = (int)(hq / hkv); p.block_size = block_size;
  p.max_blocks = (int)bt->shape[1];
  p.scale_log2 = scale * 1.4426950408889634f;

  int split = decode_split_len(S, hkv, max_ctx, max_splits, parts ? n_parts : 1);
  int n_splits = (int)((max_ctx + split - 1) / split);
  if (ws == nullptr || ws_bytes < decode_workspace_bytes(S, hkv, dv, n_splits, parts)) {
    if (parts)
      MVB_FAIL(MVB_ERR_ARG, "%s: the workspace needs %zu bytes", op, decode_workspace_bytes(S, hkv, dv, n_splits, true));
    n_splits = 1;
    split = (int)max_ctx;
  }
  p.n_splits = n_splits;
  p.split_len = split;
  p.part_o = (n_splits > 1 || parts) ? static_cast<float*>(ws) : nullptr;
  p.part_lse = p.part_o != nullptr ? p.part_o + (size_t)S * hkv * n_splits * 16 * dv : nullptr;
  p.part = parts ? part : 0;
  p.n_parts = parts ? n_parts : 1;
  p.o_part = parts ? static_cast<float*>(o->data) : nullptr;
  p.lse_part = parts ? static_cast<float*>(lse_part->data) : nullptr;
  p.n_seqs = (int)S;
  p.order = nullptr;
  // Largest-first order when the splits are long enough for the tail of the last wave to
  // outweigh the extra launch.  Config 4 steps, same box: 2.6% faster with 6.6K-token
  // splits (TP 1), 1.9% with 3.3K (TP 2), 0.8% slower with 1.7K (TP 4, context split).
  if (p.part_o != nullptr && S <= kMaxOrderedSeqs && split >= 2048) {
    const size_t pb = decode_workspace_bytes(S, hkv, dv, n_splits, parts);
    const int64_t n_own = (n_splits - p.part + p.n_parts - 1) / p.n_parts;
    if (ws_bytes >= pb + decode_order_bytes(S) && S * n_own <= 65535)
      p.order = reinterpret_cast<const int*>(static_cast<char*>(ws) + pb);
  }

  if (q->dtype == MVB_BF16) {
    switch (d) {
      case 64: launch_decode<__nv_bfloat16, 64>(p, S, st); break;
      case 128: launch_decode<__nv_bfloat16, 128>(p, S, st); break;
      case 256: launch_decode<__nv_bfloat16, 256>(p, S, st); break;
    }
  } else {
    switch (d) {
      case 64: launch_decode<__half, 64>(p, S, st); break;
      case 128: launch_decode<__half, 128>(p, S, st); break;
      case 256: launch_decode<__half, 256>(p, S, st); break;
    }
  }
  MVB_CHECK_LAUNCH(op);
  return MVB_OK;
}

}  // namespace mvb

extern "C" size_t mvb_paged_attention_decode_workspace_size(int64_t n_seqs, int64_t num_kv_heads, int64_t head_v_dim,
                                                            int64_t max_context_len) {
  // Sized for the split policy run_paged_decode uses.
  const int64_t hkv = num_kv_heads;
  if (n_seqs <= 0 || hkv <= 0 || max_context_len <= 0) return 0;
  const int split = mvb::decode_split_len(n_seqs, hkv, max_context_len, mvb::kMaxSplits);
  const int n_splits = (int)((max_context_len + split - 1) / split);
  return mvb::decode_workspace_bytes_ordered(n_seqs, hkv, head_v_dim, n_splits);
}

extern "C" int mvb_paged_attention_decode(const mvb_tensor* q, const mvb_tensor* k_cache, const mvb_tensor* v_cache,
                                          const mvb_tensor* block_tables, const mvb_tensor* context_lens, float scale,
                                          int block_size, int64_t max_context_len, mvb_tensor* o, void* workspace,
                                          size_t workspace_bytes, void* stream) {
  return mvb::run_paged_decode("paged_attention_decode", q, k_cache, v_cache, block_tables, context_lens, scale,
                               block_size, max_context_len, o, workspace, workspace_bytes, mvb::kMaxSplits,
                               static_cast<cudaStream_t>(stream));
}

extern "C" int mvb_paged_attention_decode_gated(const mvb_tensor* q, const mvb_tensor* k_cache,
                                                const mvb_tensor* v_cache, const mvb_tensor* block_tables,
                                                const mvb_tensor* context_lens, float scale, int block_size,
                                                int64_t max_context_len, const mvb_tensor* gate, mvb_tensor* o,
                                                void* workspace, size_t workspace_bytes, void* stream) {
  if (gate == nullptr) MVB_FAIL(MVB_ERR_ARG, "paged_attention_decode_gated: gate is NULL");
  return mvb::run_paged_decode("paged_attention_decode_gated", q, k_cache, v_cache, block_tables, context_lens,
                               scale, block_size, max_context_len, o, workspace, workspace_bytes, mvb::kMaxSplits,
                               static_cast<cudaStream_t>(stream), gate);
}

// ---------------------------------------------------------------------------------------
// Context-split decode: the ranks that hold copies of one kv head (tensor parallelism past
// the number of kv heads) each attend over a share of every context.
extern "C" size_t mvb_paged_attention_decode_part_workspace_size(int64_t n_seqs, int64_t num_kv_heads,
                                                                 int64_t head_v_dim, int64_t max_context_len,
                                                                 int n_parts) {
  if (n_seqs <= 0 || num_kv_heads <= 0 || max_context_len <= 0 || n_parts < 1) return 0;
  const int split = mvb::decode_split_len(n_seqs, num_kv_heads, max_context_len, mvb::kMaxSplits, n_parts);
  const int n_splits = (int)((max_context_len + split - 1) / split);
  return mvb::decode_workspace_bytes_ordered(n_seqs, num_kv_heads, head_v_dim, n_splits, true);
}

extern "C" int mvb_paged_attention_decode_part(const mvb_tensor* q, const mvb_tensor* k_cache,
                                               const mvb_tensor* v_cache, const mvb_tensor* block_tables,
                                               const mvb_tensor* context_lens, float scale, int block_size,
                                               int64_t max_context_len, int part, int n_parts, mvb_tensor* o_part,
                                               mvb_tensor* lse_part, void* workspace, size_t workspace_bytes,
                                               void* stream) {
  if (lse_part == nullptr) MVB_FAIL(MVB_ERR_ARG, "paged_attention_decode_part: lse_part is NULL");
  return mvb::run_paged_decode("paged_attention_decode_part", q, k_cache, v_cache, block_tables, context_lens, scale,
                               block_size, max_context_len, o_part, workspace, workspace_bytes, mvb::kMaxSplits,
                               static_cast<cudaStream_t>(stream), nullptr, part, n_parts, lse_part);
}

extern "C" int mvb_attention_merge_parts(const mvb_tensor* o_part, const mvb_tensor* lse_parts, int part,
                                         const mvb_tensor* gate, mvb_tensor* o, void* stream) {
  using namespace mvb;
  const char* op = "attention_merge_parts";
  int rc;
  if ((rc = check_tensor(o_part, op, "o_part", 3)) || (rc = check_tensor(lse_parts, op, "lse_parts", 3)) ||
      (rc = check_tensor(o, op, "o", 3)) || (gate && (rc = check_tensor(gate, op, "gate", 3))))
    return rc;
  const int64_t S = o_part->shape[0], hq = o_part->shape[1], d = o_part->shape[2];
  const int n_parts = (int)lse_parts->shape[0];
  MVB_CHECK_ARG(o_part->dtype == MVB_F32 && lse_parts->dtype == MVB_F32, "%s: o_part and lse_parts must be fp32", op);
  MVB_CHECK_ARG(lse_parts->shape[1] == S && lse_parts->shape[2] == hq, "%s: lse_parts must be [n_parts, S, Hq]", op);
  MVB_CHECK_ARG(part >= 0 && part < n_parts, "%s: part %d of %d", op, part, n_parts);
  MVB_CHECK_ARG(o->shape[0] == S && o->shape[1] == hq && o->shape[2] == d &&
                    (o->dtype == MVB_BF16 || o->dtype == MVB_F16),
                "%s: o must be [S, Hq, Dv] bf16 or fp16", op);
  MVB_CHECK_ARG(!gate || (gate->shape[0] == S && gate->shape[1] == hq && gate->shape[2] == d &&
                          gate->dtype == o->dtype),
                "%s: gate must be [S, Hq, Dv] in the dtype of o", op);
  MVB_CHECK_SUPPORTED(d == 64 || d == 128 || d == 256, "%s: head dim must be 64, 128 or 256", op);
  MVB_CHECK_SUPPORTED(o_part->stride[0] == hq * d && o_part->stride[1] == d && o_part->stride[2] == 1 &&
                          lse_parts->stride[1] == hq && lse_parts->stride[2] == 1 && o->stride[2] == 1 &&
                          (!gate || gate->stride[2] == 1) && S <= 65535,
                      "%s: o_part and the rows of lse_parts must be contiguous", op);
  if (S == 0 || hq == 0) return MVB_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const dim3 grid((unsigned)hq, (unsigned)S);
  const float* op_ = static_cast<const float*>(o_part->data);
  const float* lp = static_cast<const float*>(lse_parts->data);
  const int64_t sg_s = gate ? gate->stride[0] : 0, sg_h = gate ? gate->stride[1] : 0;
#define MVB_MERGE_CASE(T, DD)                                                                                     \
  attention_parts_merge_kernel<T, DD><<<grid, 128, 0, st>>>(op_, lp, lse_parts->stride[0], n_parts, part,        \
                                                           gate ? static_cast<const T*>(gate->data) : nullptr,  \
                                                           sg_s, sg_h, static_cast<T*>(o->data), o->stride[0],   \
                                                           o->stride[1], (int)hq)
  if (o->dtype == MVB_BF16) {
    if (d == 64) MVB_MERGE_CASE(__nv_bfloat16, 64);
    else if (d == 128) MVB_MERGE_CASE(__nv_bfloat16, 128);
    else MVB_MERGE_CASE(__nv_bfloat16, 256);
  } else {
    if (d == 64) MVB_MERGE_CASE(__half, 64);
    else if (d == 128) MVB_MERGE_CASE(__half, 128);
    else MVB_MERGE_CASE(__half, 256);
  }
#undef MVB_MERGE_CASE
  MVB_CHECK_LAUNCH(op);
  return MVB_OK;
}

// ---------------------------------------------------------------------------------------
// Allocation-free paged decode.
//
// Some callers cannot allocate device memory at the point where they decode: a host
// runtime that owns all device memory and hands a plugin only the tensors it needs, or a
// latency-critical step where the allocator may synchronise the device.  This entry point
// needs no workspace: the split-KV partial results go to a fixed array that is part of the
// library's device image (every GPU that loads the library holds these 16 MiB until the
// process exits).  It splits a context only as far as the array holds the partials of
// every (sequence, kv head); when not even two splits fit it runs unsplit, which needs no
// scratch at all, exactly as the workspace entry point does without a workspace.  Nothing
// in the array has to start at zero: each call writes every partial it later reads.  All
// calls share the one array, so calls whose kernels overlap on the GPU (e.g. on two
// streams) race; issue them in order.
namespace mvb {
namespace {

constexpr size_t kDecodeScratchBytes = size_t(16) << 20;
static __device__ __align__(256) char g_decode_scratch[kDecodeScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_decode_scratch_mu;
void* g_decode_scratch_addr[kMaxDevices] = {};

// Device address of g_decode_scratch on the current device.  The first call on a device
// looks it up (cudaGetSymbolAddress); later calls reuse it.
int decode_scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) MVB_FAIL(MVB_ERR_CUDA, "paged_attention_decode_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) MVB_FAIL(MVB_ERR_UNSUPPORTED, "paged_attention_decode_noalloc: device %d", dev);
  std::lock_guard<std::mutex> lock(g_decode_scratch_mu);
  if (g_decode_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_decode_scratch);
    if (e != cudaSuccess || p == nullptr)
      MVB_FAIL(MVB_ERR_CUDA, "paged_attention_decode_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    g_decode_scratch_addr[dev] = p;
  }
  *out = g_decode_scratch_addr[dev];
  return MVB_OK;
}

}  // namespace
}  // namespace mvb

extern "C" int mvb_paged_attention_decode_noalloc(const mvb_tensor* q, const mvb_tensor* k_cache,
                                                  const mvb_tensor* v_cache, const mvb_tensor* block_tables,
                                                  const mvb_tensor* context_lens, float scale, int block_size,
                                                  int64_t max_context_len, mvb_tensor* o, void* stream) {
  using namespace mvb;
  const char* op = "paged_attention_decode_noalloc";
  int rc;
  if ((rc = check_tensor(q, op, "q", 3)) || (rc = check_tensor(k_cache, op, "k_cache", 4)) ||
      (rc = check_tensor(v_cache, op, "v_cache", 4)))
    return rc;
  const int64_t S = q->shape[0], hkv = k_cache->shape[2], dv = v_cache->shape[3];
  const size_t per_split = (size_t)(S > 0 ? S : 1) * (size_t)(hkv > 0 ? hkv : 1) * 16 * (size_t)(dv + 1) * sizeof(float);
  const size_t fit = kDecodeScratchBytes / per_split;  // splits whose partials fit the array
  void* scratch = nullptr;
  if ((rc = decode_scratch_address(&scratch))) return rc;
  const int64_t max_splits = fit < 1 ? 1 : (fit < (size_t)kMaxSplits ? (int64_t)fit : (int64_t)kMaxSplits);
  return run_paged_decode(op, q, k_cache, v_cache, block_tables, context_lens, scale, block_size, max_context_len, o,
                          scratch, kDecodeScratchBytes, max_splits, static_cast<cudaStream_t>(stream));
}
