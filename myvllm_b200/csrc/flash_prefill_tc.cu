// Varlen causal flash-attention prefill on the sm_100a tensor cores (tcgen05 + TMA).
//
// Same math as flash_attention_varlen_kernel (m/ops/full_attention.py:6-111) and its paged
// variant (m/ops/full_attention.py:373-451): q-head h reads kv-head h / (Hq / Hkv), online
// softmax in fp32, optional causal mask; queries of a paged prefill sit at key positions
// ctx - L + i.
//
// One CTA = 128 query rows of one (sequence, q-head), 6 warps with fixed roles:
//   warp 0     TMA producer: Q once, then K/V tiles of 128 keys into a 1-, 2- or 3-stage
//              ring (by head dim 256, 128, 64), K_j issued ahead of V_{j-1}
//              (3-D maps [T, H, D] for contiguous K/V; 4-D maps [blocks, bs, H, D] for the
//              paged cache, one box per page segment);
//   warp 1     MMA issuer (one thread): S_j = Q K_j^T into a TMEM score buffer, then
//              O += P_{j-1} V_{j-1} into the TMEM output accumulator with P taken straight
//              from tensor memory (A operand in TMEM), so the tensor core computes the next
//              scores while the softmax warps work on this tile;
//   warps 2-5  softmax: one query row per thread (TMEM lane = row); the row's scores are
//              read into registers (which frees the score buffer at once) and its P goes
//              back into one of two TMEM P buffers as bf16/fp16 pairs; the output is
//              rescaled only when a row maximum grows by more than 2^8 (the final 1/l
//              normalisation absorbs the stale maximum), then the epilogue.
// TMEM (512 columns): O in [0, D), NSB score buffers of BN columns, two P buffers of BN/2
// columns.  P never touches shared memory: no P stores, no P operand reads.
// Every wait is bounded; a wait that gives up sets the device error word and the CTA
// drains its copies, frees TMEM and exits.
#include "flash_prefill.cuh"
#include "tcgen05.cuh"
#include "tma.cuh"

namespace mvb {
namespace {

using namespace umma;

// keys per K/V tile: 128, so each score MMA is 128 x 128 (narrower tiles leave the tensor
// pipe idle between short MMAs); the host's paged-layout check uses the same number
constexpr int fa_tc_bn(int) { return 128; }

template <int D>
struct FaTc {
  static constexpr int BM = 128;
  // what fits in 227 KB next to Q: at D = 256 one K/V stage
  static constexpr int BN = fa_tc_bn(D);
  static constexpr int NS = D == 256 ? 1 : D == 128 ? 3 : 4;  // K/V ring stages
  static constexpr int NSB = D == 256 ? 1 : 2;                // TMEM score buffers
  static constexpr int DB = D / 64;
  static constexpr uint32_t Q_BYTES = BM * D * 2;
  static constexpr uint32_t KV_BYTES = BN * D * 2;
  static constexpr uint32_t OFF_K = Q_BYTES;
  static constexpr uint32_t OFF_V = OFF_K + NS * KV_BYTES;
  static constexpr uint32_t OFF_BAR = OFF_V + NS * KV_BYTES;
  static constexpr uint32_t SMEM = OFF_BAR + 256 + 1024;
  // TMEM columns: O, the score buffers, the two P buffers
  static constexpr uint32_t COL_S = D, COL_P = D + NSB * BN;
  static_assert(SMEM <= 232448, "shared memory budget");
  static_assert(COL_P + 2 * (BN / 2) <= 512, "TMEM budget");
};

struct FaBars {
  uint64_t q_full;
  uint64_t k_full[4], k_empty[4], v_full[4], v_empty[4];
  uint64_t s_full[2], s_free[2], p_full[2], p_free[2];
  uint64_t o_done;
  uint32_t tmem_base;
};

struct FaTcParams {
  CUtensorMap tm_q, tm_k, tm_v;
  void* o;
  const int32_t* cu;
  const int32_t* bt;
  const int32_t* ctx;
  int64_t so_t, so_h, sbt_s, sbt_b;
  int n_seqs, hq, hkv, causal, block_size, page_rows;
  float scale_log2;
};

constexpr int kThreads = 192;
constexpr int kErrFa = 3;

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// Warp-uniform bounded wait: every lane polls, the warp agrees on the outcome.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t phase) {
  return __all_sync(0xffffffffu, mbar_wait(bar, phase));
}

template <typename T, int D, bool PAGED>
__global__ void __launch_bounds__(kThreads, 1) fa_tc_kernel(const __grid_constant__ FaTcParams p) {
  using C = FaTc<D>;
  constexpr int BM = C::BM, BN = C::BN, NS = C::NS, NSB = C::NSB, DB = C::DB;
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  extern __shared__ __align__(1024) char smem_raw[];
  char* smem = align1024(smem_raw);
  FaBars* bars = reinterpret_cast<FaBars*>(smem + C::OFF_BAR);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  int seq, q0;
  if (!map_query_tile<BM>(p.cu, p.n_seqs, blockIdx.y, seq, q0)) return;
  const int h = blockIdx.x;
  const int kvh = h / (p.hq / p.hkv);
  const int start = p.cu[seq];
  const int L = p.cu[seq + 1] - start;
  const int kv_len = PAGED ? p.ctx[seq] : L;
  const int qoff = PAGED ? kv_len - L : 0;
  const int kv_end = p.causal ? max(0, min(kv_len, qoff + q0 + BM)) : kv_len;
  const int n_tiles = (kv_end + BN - 1) / BN;

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    for (int s = 0; s < NS; ++s) {
      mbar_init(&bars->k_full[s], 1);
      mbar_init(&bars->k_empty[s], 1);
      mbar_init(&bars->v_full[s], 1);
      mbar_init(&bars->v_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars->s_full[s], 1);
      mbar_init(&bars->s_free[s], 4);
      mbar_init(&bars->p_full[s], 4);
      mbar_init(&bars->p_free[s], 1);
    }
    mbar_init(&bars->o_done, 1);
    mbar_fence_init();
  }
  if (warp == 1) tmem_alloc(&bars->tmem_base, 512);
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = bars->tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0 && n_tiles > 0) {
      tma::prefetch_map(&p.tm_q);
      tma::prefetch_map(&p.tm_k);
      tma::prefetch_map(&p.tm_v);
      tma::expect_tx(&bars->q_full, C::Q_BYTES);
      for (int b = 0; b < DB; ++b)
        tma::load_3d((smem + b * BM * 128), &p.tm_q, b * 64, h, start + q0, &bars->q_full);
      // one K or V tile: DB column blocks of [BN keys][64 dims]
      auto load_tile = [&](const CUtensorMap* map, char* dst, int j0, uint64_t* bar) {
        tma::expect_tx(bar, C::KV_BYTES);
        if constexpr (PAGED) {
          const int bs = p.block_size, rows = p.page_rows;
          const int last_page = (kv_len - 1) / bs;  // pages past the context hold no keys
          for (int g = 0; g < BN; g += rows) {
            const int key = j0 + g;
            const int page = min(key / bs, last_page);
            const int blk = p.bt[(int64_t)seq * p.sbt_s + (int64_t)page * p.sbt_b];
            for (int b = 0; b < DB; ++b)
              tma::load_4d((dst + b * BN * 128 + g * 128), map, b * 64, kvh, key % bs, blk, bar);
          }
        } else {
          for (int b = 0; b < DB; ++b)
            tma::load_3d((dst + b * BN * 128), map, b * 64, kvh, start + j0, bar);
        }
      };
      int k_issued = 0, v_issued = 0;
      bool ok = true;
      // K_j goes out before V_{j-1}: with one stage, V_{j-1} waits for PV_{j-2}, and the
      // scores of tile j must not wait behind it
      auto load_v = [&](int i) -> bool {
        const int s = i % NS;
        if (i >= NS && !mbar_wait(&bars->v_empty[s], ((i / NS) & 1) ^ 1)) return false;
        load_tile(&p.tm_v, smem + C::OFF_V + s * C::KV_BYTES, i * BN, &bars->v_full[s]);
        v_issued = i + 1;
        return true;
      };
      for (int j = 0; j < n_tiles; ++j) {
        const int s = j % NS;
        if (j >= NS && !(ok = mbar_wait(&bars->k_empty[s], ((j / NS) & 1) ^ 1))) break;
        load_tile(&p.tm_k, smem + C::OFF_K + s * C::KV_BYTES, j * BN, &bars->k_full[s]);
        k_issued = j + 1;
        if (j >= 1 && !(ok = load_v(j - 1))) break;
      }
      if (ok) ok = load_v(n_tiles - 1);
      if (!ok) report_device_error(kErrFa);
      // drain: the copies of the last tiles must have landed before the CTA exits
      mbar_wait(&bars->q_full, 0);
      for (int j = max(0, k_issued - NS); j < k_issued; ++j) mbar_wait(&bars->k_full[j % NS], (j / NS) & 1);
      for (int j = max(0, v_issued - NS); j < v_issued; ++j) mbar_wait(&bars->v_full[j % NS], (j / NS) & 1);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------- MMA issuer
    if (lane == 0 && n_tiles > 0) {
      const uint32_t id_s = idesc_f16(BM, BN, false, false, false, kBf16);
      const uint32_t id_o = idesc_f16(BM, D, false, true, false, kBf16);
      const uint32_t qa = smem_u32(smem);
      auto issue_pv = [&](int i) -> bool {
        const int s = i % NS;
        if (!mbar_wait(&bars->v_full[s], (i / NS) & 1)) return false;
        if (!mbar_wait(&bars->p_full[i & 1], (i >> 1) & 1)) return false;
        fence_after();
        const uint32_t pa = tmem + C::COL_P + (i & 1) * (BN / 2);  // P_i: lane = row, 2 keys per column
        const uint32_t va = smem_u32(smem + C::OFF_V + s * C::KV_BYTES);
#pragma unroll
        for (int ks = 0; ks < BN / 16; ++ks)
          mma_f16_ts(tmem, pa + ks * 8, desc_mnmajor(va, BN * 128, ks), id_o, i > 0 || ks > 0);
        commit(&bars->p_free[i & 1]);
        commit(&bars->v_empty[s]);
        return true;
      };
      bool ok = mbar_wait(&bars->q_full, 0);
      for (int j = 0; j < n_tiles && ok; ++j) {
        const int s = j % NS;
        ok = mbar_wait(&bars->k_full[s], (j / NS) & 1);
        if (ok && j >= NSB) ok = mbar_wait(&bars->s_free[j % NSB], ((j - NSB) / NSB) & 1);
        if (!ok) break;
        fence_after();
        const uint32_t ka = smem_u32(smem + C::OFF_K + s * C::KV_BYTES);
        const uint32_t sc = tmem + C::COL_S + (j % NSB) * BN;
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) mma_f16(sc, desc_kmajor(qa, BM, ks), desc_kmajor(ka, BN, ks), id_s, ks > 0);
        commit(&bars->s_full[j % NSB]);
        commit(&bars->k_empty[s]);
        if (j >= 1) ok = issue_pv(j - 1);
      }
      if (ok) ok = issue_pv(n_tiles - 1);
      if (ok) commit(&bars->o_done);
      else report_device_error(kErrFa);
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------------------- softmax
    const int quad = warp & 3;
    const int r = quad * 32 + lane;  // tile row = TMEM lane
    const int qi = q0 + r;
    const int pos = qoff + qi;
    const uint32_t lt = tmem + ((uint32_t)(quad * 32) << 16);
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_tiles; ++j) {
      if (!(ok = warp_wait(&bars->s_full[j % NSB], (j / NSB) & 1))) break;
      fence_after();
      float x[BN];
#pragma unroll
      for (int c = 0; c < BN; c += 16) tmem_ld16(lt + C::COL_S + (j % NSB) * BN + c, x + c);
      tmem_wait_ld();
      fence_before();
      __syncwarp();
      if (lane == 0) tma::arrive(&bars->s_free[j % NSB]);

      const int j0 = j * BN;
      const bool need_mask = (j0 + BN > kv_len) || (p.causal && j0 + BN - 1 > qoff + q0);
      // the scale is positive, so the row maximum is taken on the raw scores and the scale
      // folds into one FFMA per element; four partial maxima / sums keep the dependent
      // chains short (each softmax warp is alone on its scheduler)
      if (need_mask) {
#pragma unroll
        for (int c = 0; c < BN; ++c)
          if (j0 + c >= kv_len || (p.causal && j0 + c > pos)) x[c] = -INFINITY;
      }
      float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int c = 0; c < BN; ++c) mx4[c & 3] = fmaxf(mx4[c & 3], x[c]);
      const float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3])) * p.scale_log2;
      const float m_new = fmaxf(m, mx);
      const bool grow = m_new > m + 8.f;
      if (j > 0 && __any_sync(0xffffffffu, grow)) {
        // rescale this warp's output rows once PV_{j-1} has landed
        if (!(ok = warp_wait(&bars->p_free[(j - 1) & 1], ((j - 1) >> 1) & 1))) break;
        fence_after();
        const float f = grow ? ex2(m - m_new) : 1.f;
#pragma unroll 1
        for (int c = 0; c < D; c += 16) {
          float o[16];
          tmem_ld16(lt + c, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) o[i] *= f;
          tmem_st16(lt + c, o);
        }
        tmem_wait_st();
        l *= f;
      }
      if (grow) m = m_new;
      const float nbase = m == -INFINITY ? 0.f : -m;
      // P_j into TMEM P buffer j & 1, once PV_{j-2} has read it
      if (j >= 2 && !(ok = warp_wait(&bars->p_free[j & 1], ((j - 2) >> 1) & 1))) break;
      const uint32_t pt = lt + C::COL_P + (j & 1) * (BN / 2);
      float rs4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int c32 = 0; c32 < BN / 32; ++c32) {
        uint32_t pk[16];
#pragma unroll
        for (int c8 = 0; c8 < 4; ++c8) {
          float e[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            e[i] = ex2(fmaf(x[c32 * 32 + c8 * 8 + i], p.scale_log2, nbase));
            rs4[i & 3] += e[i];
          }
          const uint4 u = pack8<T>(e);  // element 2t in the low half of word t
          pk[c8 * 4] = u.x;
          pk[c8 * 4 + 1] = u.y;
          pk[c8 * 4 + 2] = u.z;
          pk[c8 * 4 + 3] = u.w;
        }
        tmem_st16(pt + c32 * 16, reinterpret_cast<const float*>(pk));
      }
      const float rs = (rs4[0] + rs4[1]) + (rs4[2] + rs4[3]);
      l += rs;
      tmem_wait_st();
      fence_before();
      __syncwarp();
      if (lane == 0) tma::arrive(&bars->p_full[j & 1]);
    }
    if (ok && n_tiles > 0) ok = warp_wait(&bars->o_done, 0);
    if (ok) {
      fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      T* go = static_cast<T*>(p.o) + (int64_t)(start + qi) * p.so_t + (int64_t)h * p.so_h;
#pragma unroll 1
      for (int c = 0; c < D; c += 16) {
        float o[16];
        if (n_tiles > 0) {
          tmem_ld16(lt + c, o);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) o[i] = 0.f;
        }
#pragma unroll
        for (int i = 0; i < 16; ++i) o[i] *= inv;
        if (qi < L) {
          *reinterpret_cast<uint4*>(go + c) = pack8<T>(o);
          *reinterpret_cast<uint4*>(go + c + 8) = pack8<T>(o + 8);
        }
      }
    } else {
      report_device_error(kErrFa);
    }
  }

  fence_before();
  __syncthreads();
  if (warp == 1) {
    fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------------------ host side ----
template <typename T, int D, bool PAGED>
int launch_typed(const FaParams& fp, int64_t T_q, int64_t n_tokens_kv, int64_t n_blocks, cudaStream_t st) {
  using C = FaTc<D>;
  FaTcParams p;
  memset(&p, 0, sizeof(p));
  const int dtype = std::is_same<T, __nv_bfloat16>::value ? MVB_BF16 : MVB_F16;
  {
    const cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)fp.hq, (cuuint64_t)T_q};
    const cuuint64_t str[2] = {(cuuint64_t)fp.sq_h * 2, (cuuint64_t)fp.sq_t * 2};
    const cuuint32_t box[3] = {64, 1, (cuuint32_t)C::BM};
    if (!tma::encode(&p.tm_q, dtype, 3, fp.q, dims, str, box)) return -1;
  }
  if constexpr (PAGED) {
    const int rows = fp.block_size < C::BN ? fp.block_size : C::BN;
    const cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)fp.hkv, (cuuint64_t)fp.block_size, (cuuint64_t)n_blocks};
    const cuuint64_t sk[3] = {(cuuint64_t)fp.sk_h * 2, (cuuint64_t)fp.sk_t * 2, (cuuint64_t)fp.sk_b * 2};
    const cuuint64_t sv[3] = {(cuuint64_t)fp.sv_h * 2, (cuuint64_t)fp.sv_t * 2, (cuuint64_t)fp.sv_b * 2};
    const cuuint32_t box[4] = {64, 1, (cuuint32_t)rows, 1};
    if (!tma::encode(&p.tm_k, dtype, 4, fp.k, dims, sk, box) || !tma::encode(&p.tm_v, dtype, 4, fp.v, dims, sv, box)) return -1;
    p.page_rows = rows;
  } else {
    const cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)fp.hkv, (cuuint64_t)n_tokens_kv};
    const cuuint64_t sk[2] = {(cuuint64_t)fp.sk_h * 2, (cuuint64_t)fp.sk_t * 2};
    const cuuint64_t sv[2] = {(cuuint64_t)fp.sv_h * 2, (cuuint64_t)fp.sv_t * 2};
    const cuuint32_t box[3] = {64, 1, (cuuint32_t)C::BN};
    if (!tma::encode(&p.tm_k, dtype, 3, fp.k, dims, sk, box) || !tma::encode(&p.tm_v, dtype, 3, fp.v, dims, sv, box)) return -1;
    p.page_rows = C::BN;
  }
  p.o = fp.o;
  p.cu = fp.cu;
  p.bt = fp.bt;
  p.ctx = fp.ctx;
  p.so_t = fp.so_t;
  p.so_h = fp.so_h;
  p.sbt_s = fp.sbt_s;
  p.sbt_b = fp.sbt_b;
  p.n_seqs = fp.n_seqs;
  p.hq = fp.hq;
  p.hkv = fp.hkv;
  p.causal = fp.causal;
  p.block_size = fp.block_size;
  p.scale_log2 = fp.scale_log2;
  static unsigned long long attr_mask = 0;
  ensure_smem_attr(fa_tc_kernel<T, D, PAGED>, C::SMEM, attr_mask);
  dim3 grid(fp.hq, (unsigned)((T_q + C::BM - 1) / C::BM + fp.n_seqs));
  fa_tc_kernel<T, D, PAGED><<<grid, kThreads, C::SMEM, st>>>(p);
  return MVB_OK;
}

template <typename T, bool PAGED>
int launch_d(int d, const FaParams& p, int64_t T_q, int64_t n_kv, int64_t nb, cudaStream_t st) {
  switch (d) {
    case 64: return launch_typed<T, 64, PAGED>(p, T_q, n_kv, nb, st);
    case 128: return launch_typed<T, 128, PAGED>(p, T_q, n_kv, nb, st);
    case 256: return launch_typed<T, 256, PAGED>(p, T_q, n_kv, nb, st);
  }
  return -1;
}

bool aligned_stride(int64_t s) { return s % 8 == 0; }

}  // namespace

// Returns -1 (with *why set) when the tensor-core kernel does not take this problem.
int launch_fa_tc(const FaParams& p, int dtype, int d, bool paged, int64_t T_q, int64_t n_tokens_kv, int64_t n_blocks,
                 cudaStream_t st, const char** why) {
  auto reject = [&](const char* r) {
    *why = r;
    return -1;
  };
  if (d != 64 && d != 128 && d != 256) return reject("head dim not 64, 128 or 256");
  if (dtype != MVB_BF16 && dtype != MVB_F16) return reject("dtype not bf16/fp16");
  if (!(p.scale_log2 > 0.f)) return reject("non-positive softmax scale");  // folded into one FFMA
  // TMA: 16-byte aligned bases and strides; vectorised epilogue: 16-byte output rows
  if (!aligned16(p.q) || !aligned16(p.k) || !aligned16(p.v) || !aligned16(p.o))
    return reject("a q/k/v/o base pointer is not 16-byte aligned");
  if (!aligned_stride(p.sq_t) || !aligned_stride(p.sq_h) || !aligned_stride(p.sk_t) || !aligned_stride(p.sk_h) ||
      !aligned_stride(p.sv_t) || !aligned_stride(p.sv_h) || !aligned_stride(p.so_t) || !aligned_stride(p.so_h))
    return reject("a token or head stride is not a multiple of 8 elements");
  if (paged) {
    const int bn = fa_tc_bn(d);
    const int bs = p.block_size;
    // a K/V tile is one page segment (bs >= BN) or whole pages of >= 8 rows (bs < BN)
    const bool tiles_ok = bs >= bn ? bs % bn == 0 : (bn % bs == 0 && bs % 8 == 0);
    if (!tiles_ok) return reject("block size does not tile into the kernel's 128-key K/V tiles");
    if (!aligned_stride(p.sk_b) || !aligned_stride(p.sv_b) || n_blocks <= 0)
      return reject("cache block stride not a multiple of 8 elements, or an empty cache");
  }
  *why = "";
  if (dtype == MVB_BF16)
    return paged ? launch_d<__nv_bfloat16, true>(d, p, T_q, n_tokens_kv, n_blocks, st)
                 : launch_d<__nv_bfloat16, false>(d, p, T_q, n_tokens_kv, n_blocks, st);
  return paged ? launch_d<__half, true>(d, p, T_q, n_tokens_kv, n_blocks, st)
               : launch_d<__half, false>(d, p, T_q, n_tokens_kv, n_blocks, st);
}

}  // namespace mvb
