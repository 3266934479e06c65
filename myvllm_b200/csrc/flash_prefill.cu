// Varlen (causal) flash attention for prefill, GQA, head dim 64/128/256: the mma.sync kernel
// for layouts the tcgen05 kernel (flash_prefill_tc.cu) does not take, e.g. paged caches whose
// block size does not tile into its K/V tiles or outputs without 16-byte rows.
//
// Replaces flash_attention_varlen_kernel (m/ops/full_attention.py:6-111): same math
// (online softmax in fp32, q-head h reads kv-head h / (Hq / Hkv), optional causal mask),
// without its host sync (:142) and with the causal loop stopping at the diagonal.
//
// CTA = 128 query rows of one (sequence, q-head): 8 warps x 16 rows.  K/V tiles of 64
// tokens stream through a double-buffered, XOR-swizzled shared-memory ring (16-byte
// cp.async); QK^T and PV run on mma.sync m16n8k16 with fp32 accumulators; P stays in
// registers as the A operand of PV.  The grid is (Hq, tiles): the Hq CTAs of one query
// tile are adjacent in launch order so their shared K/V tiles are L2 hits; tiles are
// numbered per sequence on device (no host sync) and the last (most expensive under the
// causal mask) query tiles of each sequence are issued first.
#include "flash_prefill.cuh"

namespace mvb {
namespace {

constexpr int BM = 128;
constexpr int BN = 64;
constexpr int kWarps = 8;

template <int D>
__device__ __forceinline__ int swz(int r, int c) {
  return r * (D * 2) + ((c ^ (r & 7)) << 4);
}

// PAGED: queries of sequence s sit at positions ctx[s] - L_s + i and attend to the
// first ctx[s] tokens of the paged cache (reference kernel m/ops/full_attention.py:373-451).
template <typename T, int D, bool PAGED>
__global__ void __launch_bounds__(kWarps * 32, 1) flash_prefill_kernel(FaParams p) {
  constexpr int ROWB = D * 2;
  constexpr int CH = D / 8;
  constexpr int KV_BYTES = BN * ROWB;
  extern __shared__ __align__(128) char smem[];
  char* sQ = smem;                   // [BM][D]
  char* sKV = smem + BM * ROWB;      // 2 stages x (K [BN][D], V [BN][D])

  int seq, q0;
  if (!map_query_tile<BM>(p.cu, p.n_seqs, blockIdx.y, seq, q0)) return;
  const int h = blockIdx.x;
  const int kvh = h / (p.hq / p.hkv);
  const int start = p.cu[seq];
  const int L = p.cu[seq + 1] - start;               // queries of this sequence
  const int kv_len = PAGED ? p.ctx[seq] : L;         // keys it may attend to
  const int qoff = PAGED ? kv_len - L : 0;            // position of query 0 among the keys
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const T* gq = static_cast<const T*>(p.q);
  const T* gk = static_cast<const T*>(p.k);
  const T* gv = static_cast<const T*>(p.v);

  for (int i = tid; i < BM * CH; i += kWarps * 32) {
    const int r = i / CH, c = i % CH;
    const bool ok = q0 + r < L;
    cp_async16(sQ + swz<D>(r, c), gq + (int64_t)(start + (ok ? q0 + r : 0)) * p.sq_t + h * p.sq_h + c * 8, ok);
  }
  const int kv_end = p.causal ? max(0, min(kv_len, qoff + q0 + BM)) : kv_len;
  const int n_tiles = (kv_end + BN - 1) / BN;
  auto load_kv = [&](int stage, int j0) {
    char* sK = sKV + stage * 2 * KV_BYTES;
    char* sV = sK + KV_BYTES;
    for (int i = tid; i < BN * CH; i += kWarps * 32) {
      const int r = i / CH, c = i % CH;
      const bool ok = j0 + r < kv_len;
      int64_t koff, voff;
      if constexpr (PAGED) {
        const int t = ok ? j0 + r : 0;
        const int64_t blk = ok ? p.bt[seq * p.sbt_s + (t / p.block_size) * p.sbt_b] : 0;
        koff = blk * p.sk_b + (t % p.block_size) * p.sk_t + kvh * p.sk_h;
        voff = blk * p.sv_b + (t % p.block_size) * p.sv_t + kvh * p.sv_h;
      } else {
        const int64_t t = start + (ok ? j0 + r : 0);
        koff = t * p.sk_t + kvh * p.sk_h;
        voff = t * p.sv_t + kvh * p.sv_h;
      }
      cp_async16(sK + swz<D>(r, c), gk + koff + c * 8, ok);
      cp_async16(sV + swz<D>(r, c), gv + voff + c * 8, ok);
    }
  };
  load_kv(0, 0);
  cp_async_commit();

  float acc[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  const int row0 = q0 + warp * 16 + (lane >> 2), row1 = row0 + 8;  // query index in the sequence
  const int pos0 = qoff + row0, pos1 = qoff + row1;                    // its key position

  for (int it = 0; it < n_tiles; ++it) {
    const int stage = it & 1;
    if (it + 1 < n_tiles) load_kv(stage ^ 1, (it + 1) * BN);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const char* sK = sKV + stage * 2 * KV_BYTES;
    const char* sV = sK + KV_BYTES;
    const int j0 = it * BN;

    float s[BN / 8][4];
#pragma unroll
    for (int i = 0; i < BN / 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
    // skip the MMAs of warps whose 16 rows lie entirely above this tile's diagonal
    const bool live = !p.causal || (qoff + q0 + warp * 16 + 15 >= j0);
    if (live) {
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        uint32_t a[4];
        {
          const int r = warp * 16 + (lane & 15), c = kk * 2 + (lane >> 4);
          ldmatrix_x4(a[0], a[1], a[2], a[3], smem_u32(sQ + swz<D>(r, c)));
        }
#pragma unroll
        for (int np = 0; np < BN / 16; ++np) {
          uint32_t b[4];
          const int r = np * 16 + (lane & 7) + ((lane >> 4) << 3);
          const int c = kk * 2 + ((lane >> 3) & 1);
          ldmatrix_x4(b[0], b[1], b[2], b[3], smem_u32(sK + swz<D>(r, c)));
          mma16816<T>(s[np * 2], a, b);
          mma16816<T>(s[np * 2 + 1], a, b + 2);
        }
      }
    }
    const bool need_mask = (j0 + BN > kv_len) || (p.causal && j0 + BN - 1 > qoff + q0 + warp * 16);
#pragma unroll
    for (int nf = 0; nf < BN / 8; ++nf)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int j = j0 + nf * 8 + (lane & 3) * 2 + (e & 1);
        const int i = e < 2 ? pos0 : pos1;
        float x = s[nf][e] * p.scale_log2;
        if (need_mask && (j >= kv_len || (p.causal && j > i) || !live)) x = -INFINITY;
        s[nf][e] = x;
      }
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int nf = 0; nf < BN / 8; ++nf) {
      mx0 = fmaxf(mx0, fmaxf(s[nf][0], s[nf][1]));
      mx1 = fmaxf(mx1, fmaxf(s[nf][2], s[nf][3]));
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float nm0 = fmaxf(m0, mx0), nm1 = fmaxf(m1, mx1);
    const float a0 = nm0 == -INFINITY ? 1.f : exp2f(m0 - nm0);
    const float a1 = nm1 == -INFINITY ? 1.f : exp2f(m1 - nm1);
    const float b0 = nm0 == -INFINITY ? 0.f : nm0;
    const float b1 = nm1 == -INFINITY ? 0.f : nm1;
    float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
    for (int nf = 0; nf < BN / 8; ++nf) {
      s[nf][0] = exp2f(s[nf][0] - b0);
      s[nf][1] = exp2f(s[nf][1] - b0);
      s[nf][2] = exp2f(s[nf][2] - b1);
      s[nf][3] = exp2f(s[nf][3] - b1);
      ps0 += s[nf][0] + s[nf][1];
      ps1 += s[nf][2] + s[nf][3];
    }
    l0 = l0 * a0 + ps0;
    l1 = l1 * a1 + ps1;
    m0 = nm0;
    m1 = nm1;
    if (live) {
#pragma unroll
      for (int i = 0; i < D / 8; ++i) {
        acc[i][0] *= a0; acc[i][1] *= a0; acc[i][2] *= a1; acc[i][3] *= a1;
      }
#pragma unroll
      for (int kk = 0; kk < BN / 16; ++kk) {
        uint32_t pa[4];
        pa[0] = pack2<T>(s[kk * 2][0], s[kk * 2][1]);
        pa[1] = pack2<T>(s[kk * 2][2], s[kk * 2][3]);
        pa[2] = pack2<T>(s[kk * 2 + 1][0], s[kk * 2 + 1][1]);
        pa[3] = pack2<T>(s[kk * 2 + 1][2], s[kk * 2 + 1][3]);
#pragma unroll
        for (int nn = 0; nn < D / 16; ++nn) {
          uint32_t b[4];
          const int r = kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
          const int c = nn * 2 + (lane >> 4);
          ldmatrix_x4_trans(b[0], b[1], b[2], b[3], smem_u32(sV + swz<D>(r, c)));
          mma16816<T>(acc[nn * 2], pa, b);
          mma16816<T>(acc[nn * 2 + 1], pa, b + 2);
        }
      }
    }
    __syncthreads();
  }
  cp_async_wait<0>();

  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float inv0 = l0 > 0.f ? 1.f / l0 : 0.f, inv1 = l1 > 0.f ? 1.f / l1 : 0.f;
  T* go = static_cast<T*>(p.o);
#pragma unroll
  for (int nf = 0; nf < D / 8; ++nf) {
    const int c = nf * 8 + (lane & 3) * 2;
    if (row0 < L)
      *reinterpret_cast<uint32_t*>(go + (int64_t)(start + row0) * p.so_t + h * p.so_h + c) =
          pack2<T>(acc[nf][0] * inv0, acc[nf][1] * inv0);
    if (row1 < L)
      *reinterpret_cast<uint32_t*>(go + (int64_t)(start + row1) * p.so_t + h * p.so_h + c) =
          pack2<T>(acc[nf][2] * inv1, acc[nf][3] * inv1);
  }
}

template <typename T, int D, bool PAGED>
void launch_fa(const FaParams& p, int64_t T_tokens, cudaStream_t st) {
  constexpr int smem = BM * D * 2 + 2 * 2 * BN * D * 2;
  static unsigned long long attr_mask = 0;
  ensure_smem_attr(flash_prefill_kernel<T, D, PAGED>, smem, attr_mask);
  dim3 grid(p.hq, (unsigned)((T_tokens + BM - 1) / BM + p.n_seqs));
  flash_prefill_kernel<T, D, PAGED><<<grid, kWarps * 32, smem, st>>>(p);
}

template <bool PAGED>
void dispatch_fa(int dtype, int d, const FaParams& p, int64_t T, cudaStream_t st) {
  if (dtype == MVB_BF16) {
    switch (d) {
      case 64: launch_fa<__nv_bfloat16, 64, PAGED>(p, T, st); break;
      case 128: launch_fa<__nv_bfloat16, 128, PAGED>(p, T, st); break;
      case 256: launch_fa<__nv_bfloat16, 256, PAGED>(p, T, st); break;
    }
  } else {
    switch (d) {
      case 64: launch_fa<__half, 64, PAGED>(p, T, st); break;
      case 128: launch_fa<__half, 128, PAGED>(p, T, st); break;
      case 256: launch_fa<__half, 256, PAGED>(p, T, st); break;
    }
  }
}

}  // namespace
}  // namespace mvb

extern "C" int mvb_flash_attention_prefill(const mvb_tensor* q, const mvb_tensor* k, const mvb_tensor* v,
                                           const mvb_tensor* cu_seqlens, float scale, int num_heads,
                                           int num_kv_heads, int head_dim, int head_v_dim, int is_causal,
                                           mvb_tensor* o, void* stream) {
  using namespace mvb;
  const char* op = "flash_attention_prefill";
  int rc;
  if ((rc = check_tensor(q, op, "q", 3)) || (rc = check_tensor(k, op, "k", 3)) ||
      (rc = check_tensor(v, op, "v", 3)) || (rc = check_tensor(cu_seqlens, op, "cu_seqlens", 1)) ||
      (rc = check_tensor(o, op, "o", 3)))
    return rc;
  const int64_t T = q->shape[0];
  MVB_CHECK_ARG(q->shape[1] == num_heads && q->shape[2] == head_dim, "%s: q must be [T, num_heads, head_dim]", op);
  MVB_CHECK_ARG(k->shape[0] == T && k->shape[1] == num_kv_heads && k->shape[2] == head_dim,
                "%s: k must be [T, num_kv_heads, head_dim]", op);
  MVB_CHECK_ARG(v->shape[0] == T && v->shape[1] == num_kv_heads && v->shape[2] == head_v_dim,
                "%s: v must be [T, num_kv_heads, head_v_dim]", op);
  MVB_CHECK_ARG(o->shape[0] == T && o->shape[1] == num_heads && o->shape[2] == head_v_dim, "%s: o shape", op);
  MVB_CHECK_ARG(num_kv_heads > 0 && num_heads % num_kv_heads == 0, "%s: num_heads %% num_kv_heads != 0", op);
  MVB_CHECK_ARG(cu_seqlens->dtype == MVB_I32 && cu_seqlens->shape[0] >= 1, "%s: cu_seqlens must be int32 [S+1]", op);
  MVB_CHECK_ARG(q->dtype == k->dtype && q->dtype == v->dtype && q->dtype == o->dtype, "%s: dtype mismatch", op);
  MVB_CHECK_SUPPORTED(q->dtype == MVB_BF16 || q->dtype == MVB_F16, "%s: bf16/fp16 only", op);
  MVB_CHECK_SUPPORTED(head_dim == head_v_dim && (head_dim == 64 || head_dim == 128 || head_dim == 256),
                      "%s: head_dim must equal head_v_dim and be 64, 128 or 256", op);
  MVB_CHECK_SUPPORTED(q->stride[2] == 1 && k->stride[2] == 1 && v->stride[2] == 1 && o->stride[2] == 1 &&
                          q->stride[0] % 8 == 0 && q->stride[1] % 8 == 0 && k->stride[0] % 8 == 0 &&
                          k->stride[1] % 8 == 0 && v->stride[0] % 8 == 0 && v->stride[1] % 8 == 0 &&
                          o->stride[0] % 2 == 0 && o->stride[1] % 2 == 0 && aligned16(q->data) &&
                          aligned16(k->data) && aligned16(v->data) &&
                          (reinterpret_cast<uintptr_t>(o->data) & 3) == 0,
                      "%s: rows must be contiguous and 16-byte aligned", op);
  const int64_t n_seqs = cu_seqlens->shape[0] - 1;
  MVB_CHECK_SUPPORTED(num_heads <= 65535 && (T + 127) / 128 + n_seqs <= 65535, "%s: too many heads or tokens", op);
  if (T == 0 || n_seqs == 0 || num_heads == 0) return MVB_OK;
  FaParams p;
  p.q = q->data; p.k = k->data; p.v = v->data; p.o = o->data;
  p.cu = static_cast<const int32_t*>(cu_seqlens->data);
  p.sq_t = q->stride[0]; p.sq_h = q->stride[1]; p.sk_t = k->stride[0]; p.sk_h = k->stride[1];
  p.sv_t = v->stride[0]; p.sv_h = v->stride[1]; p.so_t = o->stride[0]; p.so_h = o->stride[1];
  p.n_seqs = (int)n_seqs; p.hq = num_heads; p.hkv = num_kv_heads; p.causal = is_causal ? 1 : 0;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.bt = nullptr; p.ctx = nullptr; p.sk_b = p.sv_b = p.sbt_s = p.sbt_b = 0; p.block_size = 1;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const char* why = "";
  if (launch_fa_tc(p, q->dtype, head_dim, false, T, T, 0, st, &why) < 0) {
    set_path(MVB_OP_FA_PREFILL, MVB_PATH_MMA_SYNC, why);
    dispatch_fa<false>(q->dtype, head_dim, p, T, st);
  } else {
    set_path(MVB_OP_FA_PREFILL, MVB_PATH_TENSOR_CORE, "");
  }
  MVB_CHECK_LAUNCH(op);
  return MVB_OK;
}

extern "C" int mvb_paged_attention_prefill(const mvb_tensor* q, const mvb_tensor* k_cache, const mvb_tensor* v_cache,
                                           const mvb_tensor* block_tables, const mvb_tensor* context_lens,
                                           const mvb_tensor* cu_seqlens, float scale, int block_size, mvb_tensor* o,
                                           void* stream) {
  using namespace mvb;
  const char* op = "paged_attention_prefill";
  int rc;
  if ((rc = check_tensor(q, op, "q", 3)) || (rc = check_tensor(k_cache, op, "k_cache", 4)) ||
      (rc = check_tensor(v_cache, op, "v_cache", 4)) || (rc = check_tensor(block_tables, op, "block_tables", 2)) ||
      (rc = check_tensor(context_lens, op, "context_lens", 1)) ||
      (rc = check_tensor(cu_seqlens, op, "cu_seqlens", 1)) || (rc = check_tensor(o, op, "o", 3)))
    return rc;
  const int64_t T = q->shape[0], hq = q->shape[1], d = q->shape[2];
  const int64_t hkv = k_cache->shape[2], dv = v_cache->shape[3];
  const int64_t n_seqs = cu_seqlens->shape[0] - 1;
  MVB_CHECK_ARG(k_cache->shape[1] == block_size && v_cache->shape[1] == block_size && block_size > 0,
                "%s: caches must be [n_blocks, block_size, Hkv, D]", op);
  MVB_CHECK_ARG(k_cache->shape[3] == d && v_cache->shape[2] == hkv, "%s: cache shapes disagree with q", op);
  MVB_CHECK_ARG(hkv > 0 && hq % hkv == 0, "%s: Hq must be a multiple of Hkv", op);
  MVB_CHECK_ARG(o->shape[0] == T && o->shape[1] == hq && o->shape[2] == dv, "%s: o must be [T, Hq, Dv]", op);
  MVB_CHECK_ARG(cu_seqlens->dtype == MVB_I32 && block_tables->dtype == MVB_I32 && context_lens->dtype == MVB_I32,
                "%s: index tensors must be int32", op);
  MVB_CHECK_ARG(n_seqs >= 0 && block_tables->shape[0] >= n_seqs && context_lens->shape[0] >= n_seqs,
                "%s: block_tables/context_lens shorter than the batch", op);
  MVB_CHECK_ARG(q->dtype == k_cache->dtype && q->dtype == v_cache->dtype && q->dtype == o->dtype,
                "%s: dtype mismatch", op);
  MVB_CHECK_SUPPORTED(q->dtype == MVB_BF16 || q->dtype == MVB_F16, "%s: bf16/fp16 only", op);
  MVB_CHECK_SUPPORTED(d == dv && (d == 64 || d == 128 || d == 256), "%s: head dim must be 64, 128 or 256", op);
  MVB_CHECK_SUPPORTED(q->stride[2] == 1 && o->stride[2] == 1 && k_cache->stride[3] == 1 && v_cache->stride[3] == 1 &&
                          q->stride[0] % 8 == 0 && q->stride[1] % 8 == 0 && k_cache->stride[0] % 8 == 0 &&
                          k_cache->stride[1] % 8 == 0 && k_cache->stride[2] % 8 == 0 &&
                          v_cache->stride[0] % 8 == 0 && v_cache->stride[1] % 8 == 0 &&
                          v_cache->stride[2] % 8 == 0 && o->stride[0] % 2 == 0 && o->stride[1] % 2 == 0 &&
                          aligned16(q->data) && aligned16(k_cache->data) && aligned16(v_cache->data) &&
                          (reinterpret_cast<uintptr_t>(o->data) & 3) == 0,
                      "%s: rows must be contiguous and 16-byte aligned", op);
  MVB_CHECK_SUPPORTED(hq <= 65535 && (T + 127) / 128 + n_seqs <= 65535, "%s: too many heads or tokens", op);
  if (T == 0 || n_seqs == 0 || hq == 0) return MVB_OK;
  FaParams p;
  p.q = q->data; p.k = k_cache->data; p.v = v_cache->data; p.o = o->data;
  p.cu = static_cast<const int32_t*>(cu_seqlens->data);
  p.sq_t = q->stride[0]; p.sq_h = q->stride[1];
  p.sk_b = k_cache->stride[0]; p.sk_t = k_cache->stride[1]; p.sk_h = k_cache->stride[2];
  p.sv_b = v_cache->stride[0]; p.sv_t = v_cache->stride[1]; p.sv_h = v_cache->stride[2];
  p.so_t = o->stride[0]; p.so_h = o->stride[1];
  p.bt = static_cast<const int32_t*>(block_tables->data);
  p.ctx = static_cast<const int32_t*>(context_lens->data);
  p.sbt_s = block_tables->stride[0]; p.sbt_b = block_tables->stride[1];
  p.block_size = block_size;
  p.n_seqs = (int)n_seqs; p.hq = (int)hq; p.hkv = (int)hkv; p.causal = 1;
  p.scale_log2 = scale * 1.4426950408889634f;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const char* why = "";
  if (launch_fa_tc(p, q->dtype, (int)d, true, T, 0, k_cache->shape[0], st, &why) < 0) {
    set_path(MVB_OP_PAGED_PREFILL, MVB_PATH_MMA_SYNC, why);
    dispatch_fa<true>(q->dtype, (int)d, p, T, st);
  } else {
    set_path(MVB_OP_PAGED_PREFILL, MVB_PATH_TENSOR_CORE, "");
  }
  MVB_CHECK_LAUNCH(op);
  return MVB_OK;
}
