// Chunked gated delta rule (prefill), WY form with chunk C = 64, K = V = 128.
//
// Replaces the reference's six-launch pipeline (m/ops/gated_delta_rule/gated_delta_rule.py:44-64:
// cumsum.py -> chunk_scaled_dot_kkt.py -> solve_tril.py -> wu.py -> h.py -> o.py) with ONE
// kernel in which a CTA walks one (sequence, v-head) chain chunk by chunk and keeps every
// intermediate on chip.  HBM traffic is the algorithmic minimum: q, k, v, g, beta read once,
// o written once, the fp32 state read and written once per chain.
//
// Per chunk (n <= 64 valid rows; padded rows have beta = g = 0 and zero q/k/v):
//   G      = cumsum(g)                                   (kept as log2: G2 = G * log2 e)
//   A      = strict_lower(beta_i k_i.k_j e^{G_i-G_j})   Aqk = lower(q_i.k_j e^{G_i-G_j})
//   Ti     = (I + A)^-1  (fp32 forward substitution, one thread per column)
//   u      = (Ti diag(beta)) v,   w = (Ti diag(beta e^G)) k
//   v_new  = u - w S;   o = scale (e^G (q S) + Aqk v_new)
//   S     <- e^{G_last} S + k^T (e^{G_last - G} v_new)   (S: fp32 registers, bf16 copy in smem)
// Numerics: every contraction runs with fp16 operands and fp32 accumulation.  bf16 q/k/v
// tiles are converted to fp16 in shared memory right after they land (exact for
// 6e-5 < |x| < 65504), optionally L2-normalising q and k rows in the same pass; the
// internal operands (Ti, w, the state copy, v_new) are then rounded to fp16 (2^-11)
// instead of bf16 (2^-8), which keeps the final fp32 state within 1e-3 relative of the
// exact recurrence.  Contractions run on mma.sync m16n8k16; 8 warps, each owning a
// 16-row x 64-column slab (or 16 state rows x 128 columns for the update).
//
// Scheduling: a persistent grid; chains are handed out longest sequence first (the rank
// of each sequence is computed on device) so the longest serial chain starts at once.
#include <type_traits>

#include "common.cuh"

namespace mvb {

int check_gdn(const char* op, const mvb_tensor* q, const mvb_tensor* k, const mvb_tensor* v, const mvb_tensor* g,
              const mvb_tensor* beta, const mvb_tensor* state, const mvb_tensor* idx, const mvb_tensor* cu,
              const mvb_tensor* o, int64_t* n_seqs_out);
int run_recurrent(const char* op, const mvb_tensor* q, const mvb_tensor* k, const mvb_tensor* v,
                  const mvb_tensor* g, const mvb_tensor* beta, mvb_tensor* state, const mvb_tensor* idx,
                  const mvb_tensor* cu, mvb_tensor* o, float scale, int l2norm, cudaStream_t st);

namespace {

constexpr int C = 64;       // chunk
constexpr int KD = 128;     // k head dim
constexpr int VD = 128;     // v head dim
constexpr int kThreads = 256;
constexpr int kMaxSortSeqs = 1024;

// shared-memory map (bytes)
constexpr int OFF_Q = 0;                       // [64][128] T
constexpr int OFF_K = OFF_Q + C * KD * 2;      // [64][128] T
constexpr int OFF_V = OFF_K + C * KD * 2;      // [64][128] T
constexpr int OFF_S = OFF_V + C * VD * 2;      // [128][128] T (bf16 copy of the state)
constexpr int OFF_AW = OFF_S + KD * VD * 2;    // [64][64] f32 A  | later [64][128] T w
constexpr int OFF_T = OFF_AW + C * C * 4;      // [64][64] T Tu + [64][64] T Tw | later [64][128] T v'
constexpr int OFF_AQK = OFF_T + 2 * C * C * 2; // [64][64] T
constexpr int OFF_VN = OFF_AQK + C * C * 2;    // [64][128] T v_new
constexpr int OFF_G = OFF_VN + C * VD * 2;     // [64] f32 G2
constexpr int OFF_B = OFF_G + C * 4;           // [64] f32 beta
constexpr int OFF_PERM = OFF_B + C * 4;        // [1024] int
constexpr int SMEM_BYTES = OFF_PERM + kMaxSortSeqs * 4;

struct ChunkParams {
  const void *q, *k, *v, *g, *beta;
  void* o;
  float* state;
  const int32_t* state_idx;
  const int32_t* cu;
  int64_t sq_t, sq_h, sk_t, sk_h, sv_t, sv_h, so_t, so_h, sg_t, sg_h, sb_t, sb_h;
  int64_t ss_n, ss_h, ss_k;
  int n_seqs, hk, hv, l2norm;
  float scale;
};

// 256-byte rows (128 x 16-bit), 16 chunks of 16 bytes, XOR-swizzled.
__device__ __forceinline__ int sw256(int r, int c) { return r * 256 + ((c ^ (r & 7)) << 4); }
// 128-byte rows (64 x 16-bit).
__device__ __forceinline__ int sw128(int r, int c) { return r * 128 + ((c ^ (r & 7)) << 4); }

// Element (r, col) of a swizzled 16-bit matrix with 256- or 128-byte rows.
template <int ROWB>
__device__ __forceinline__ int elem(int r, int col) {
  if constexpr (ROWB == 256) return sw256(r, col >> 3) + ((col & 7) << 1);
  else return sw128(r, col >> 3) + ((col & 7) << 1);
}

// A fragment (16 x 16, row-major) at rows r0.., k-chunk pair kc (16 columns) of a
// swizzled matrix whose rows are ROWB bytes.
template <int ROWB>
__device__ __forceinline__ void lda(uint32_t* a, const char* base, int r0, int kc, int lane) {
  const int r = r0 + (lane & 15), c = kc * 2 + (lane >> 4);
  const int off = ROWB == 256 ? sw256(r, c) : sw128(r, c);
  ldmatrix_x4(a[0], a[1], a[2], a[3], smem_u32(base + off));
}
// A fragment of M^T where M is stored [k rows][m cols]: rows m0.. of M^T, k rows k0..k0+15.
template <int ROWB>
__device__ __forceinline__ void lda_t(uint32_t* a, const char* base, int m0, int k0, int lane) {
  const int mi = lane >> 3;
  const int r = k0 + (lane & 7) + ((mi >> 1) << 3);
  const int c = (m0 >> 3) + (mi & 1);
  const int off = ROWB == 256 ? sw256(r, c) : sw128(r, c);
  ldmatrix_x4_trans(a[0], a[1], a[2], a[3], smem_u32(base + off));
}
// Two B fragments (k16 x n16) from a matrix stored [k rows][n cols] (transposed load).
template <int ROWB>
__device__ __forceinline__ void ldb_kn(uint32_t* b, const char* base, int k0, int n0, int lane) {
  const int r = k0 + (lane & 7) + (((lane >> 3) & 1) << 3);
  const int c = (n0 >> 3) + (lane >> 4);
  const int off = ROWB == 256 ? sw256(r, c) : sw128(r, c);
  ldmatrix_x4_trans(b[0], b[1], b[2], b[3], smem_u32(base + off));
}
// Two B fragments (k16 x n16) from a matrix stored [n rows][k cols] (plain load).
template <int ROWB>
__device__ __forceinline__ void ldb_nk(uint32_t* b, const char* base, int n0, int k0, int lane) {
  const int r = n0 + (lane & 7) + ((lane >> 4) << 3);
  const int c = (k0 >> 3) + ((lane >> 3) & 1);
  const int off = ROWB == 256 ? sw256(r, c) : sw128(r, c);
  ldmatrix_x4(b[0], b[1], b[2], b[3], smem_u32(base + off));
}

template <typename T>
__device__ __forceinline__ void st2(char* base, int off, float a, float b) {
  *reinterpret_cast<uint32_t*>(base + off) = pack2<T>(a, b);
}

// In place: 16-bit input tile rows -> fp16, q/k rows optionally scaled by
// rsqrt(sum x^2 + 1e-6) (m/layers/linear_attention.py:113-114).  4 threads per row.
template <typename T>
__device__ __forceinline__ void convert_tiles(char* sQ, char* sK, char* sV, bool l2norm, int tid) {
  const int r = tid >> 2, qq = tid & 3;  // row, quarter (4 chunks of 8)
#pragma unroll
  for (int m = 0; m < 2; ++m) {
    char* base = m == 0 ? sQ : sK;
    float f[4][8];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      unpack8<T>(*reinterpret_cast<const uint4*>(base + sw256(r, qq * 4 + i)), f[i]);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += f[i][j] * f[i][j];
    }
    float sc = 1.f;
    if (l2norm) {
      ss += __shfl_xor_sync(0xffffffffu, ss, 1);
      ss += __shfl_xor_sync(0xffffffffu, ss, 2);
      sc = rsqrtf(ss + 1e-6f);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
#pragma unroll
      for (int j = 0; j < 8; ++j) f[i][j] *= sc;
      *reinterpret_cast<uint4*>(base + sw256(r, qq * 4 + i)) = pack8<__half>(f[i]);
    }
  }
  if constexpr (!std::is_same<T, __half>::value) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float f[8];
      unpack8<T>(*reinterpret_cast<const uint4*>(sV + sw256(r, qq * 4 + i)), f);
      *reinterpret_cast<uint4*>(sV + sw256(r, qq * 4 + i)) = pack8<__half>(f);
    }
  }
}

template <typename T, typename TG>
__global__ void __launch_bounds__(kThreads, 1) gdn_chunk_kernel(ChunkParams p) {
  using CT = __half;  // compute (MMA operand) type
  extern __shared__ __align__(128) char smem[];
  char* sQ = smem + OFF_Q;
  char* sK = smem + OFF_K;
  char* sV = smem + OFF_V;
  char* sS = smem + OFF_S;
  float* sA = reinterpret_cast<float*>(smem + OFF_AW);
  char* sW = smem + OFF_AW;
  char* sTu = smem + OFF_T;
  char* sTw = smem + OFF_T + C * C * 2;
  char* sVp = smem + OFF_T;
  char* sAqk = smem + OFF_AQK;
  char* sVn = smem + OFF_VN;
  float* sG = reinterpret_cast<float*>(smem + OFF_G);
  float* sB = reinterpret_cast<float*>(smem + OFF_B);
  int* sPerm = reinterpret_cast<int*>(smem + OFF_PERM);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int mt = warp & 3;     // 16-row block of a 64-row operand
  const int nh = warp >> 2;    // 64-column half
  const int qr = lane >> 2;    // fragment row within 8
  const int qc = (lane & 3) * 2;

  // Longest-sequence-first order (ties by index).
  const int S = p.n_seqs;
  const bool sorted = S <= kMaxSortSeqs;
  if (sorted) {
    for (int i = tid; i < S; i += kThreads) {
      const int li = p.cu[i + 1] - p.cu[i];
      int rank = 0;
      for (int j = 0; j < S; ++j) {
        const int lj = p.cu[j + 1] - p.cu[j];
        rank += (lj > li) || (lj == li && j < i);
      }
      sPerm[rank] = i;
    }
  }
  __syncthreads();

  const T* gq = static_cast<const T*>(p.q);
  const T* gk = static_cast<const T*>(p.k);
  const T* gv = static_cast<const T*>(p.v);
  const TG* gg = static_cast<const TG*>(p.g);
  const TG* gb = static_cast<const TG*>(p.beta);
  T* go = static_cast<T*>(p.o);
  constexpr float LOG2E = 1.4426950408889634f;

  const int n_chains = S * p.hv;
  for (int chain = blockIdx.x; chain < n_chains; chain += gridDim.x) {
    const int seq = sorted ? sPerm[chain / p.hv] : chain / p.hv;
    const int h = chain % p.hv;
    const int kh = h / (p.hv / p.hk);
    const int t_begin = p.cu[seq], t_end = p.cu[seq + 1];
    float* gstate = p.state + (int64_t)p.state_idx[seq] * p.ss_n + (int64_t)h * p.ss_h;

    // State rows [16 warp, +16) x 128 columns in registers (16 n8 fragments).
    float Sr[16][4];
#pragma unroll
    for (int nf = 0; nf < 16; ++nf) {
      const int col = nf * 8 + qc;
      const float2 lo = *reinterpret_cast<const float2*>(gstate + (warp * 16 + qr) * p.ss_k + col);
      const float2 hi = *reinterpret_cast<const float2*>(gstate + (warp * 16 + qr + 8) * p.ss_k + col);
      Sr[nf][0] = lo.x; Sr[nf][1] = lo.y; Sr[nf][2] = hi.x; Sr[nf][3] = hi.y;
      st2<CT>(sS, elem<256>(warp * 16 + qr, col), lo.x, lo.y);
      st2<CT>(sS, elem<256>(warp * 16 + qr + 8, col), hi.x, hi.y);
    }

    for (int c0 = t_begin; c0 < t_end; c0 += C) {
      const int n = min(C, t_end - c0);
      // ---- load chunk (rows >= n zero-filled) ----
      for (int i = tid; i < C * 16; i += kThreads) {
        const int r = i >> 4, c = i & 15;
        const bool ok = r < n;
        const int t = ok ? c0 + r : c0;
        cp_async16(sQ + sw256(r, c), gq + t * p.sq_t + kh * p.sq_h + c * 8, ok);
        cp_async16(sK + sw256(r, c), gk + t * p.sk_t + kh * p.sk_h + c * 8, ok);
        cp_async16(sV + sw256(r, c), gv + t * p.sv_t + h * p.sv_h + c * 8, ok);
      }
      cp_async_commit();
      if (warp == 0) {
        // G2 = cumsum(g) * log2(e); each lane owns rows 2 lane, 2 lane + 1
        const int r0 = 2 * lane, r1 = r0 + 1;
        const float g0 = r0 < n ? to_f32<TG>(gg[(c0 + r0) * p.sg_t + h * p.sg_h]) : 0.f;
        const float g1 = r1 < n ? to_f32<TG>(gg[(c0 + r1) * p.sg_t + h * p.sg_h]) : 0.f;
        float incl = g0 + g1;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const float y = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= o) incl += y;
        }
        const float excl = incl - (g0 + g1);
        sG[r0] = (excl + g0) * LOG2E;
        sG[r1] = incl * LOG2E;
        sB[r0] = r0 < n ? to_f32<TG>(gb[(c0 + r0) * p.sb_t + h * p.sb_h]) : 0.f;
        sB[r1] = r1 < n ? to_f32<TG>(gb[(c0 + r1) * p.sb_t + h * p.sb_h]) : 0.f;
      }
      cp_async_wait<0>();
      __syncthreads();
      convert_tiles<T>(sQ, sK, sV, p.l2norm != 0, tid);
      __syncthreads();

      // ---- step 1: A = k k^T, Aqk = q k^T  (warp: rows 16 mt, cols 32 nh) ----
      {
        float akk[4][4], aqk[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) akk[i][j] = aqk[i][j] = 0.f;
#pragma unroll
        for (int kc = 0; kc < KD / 16; ++kc) {
          uint32_t ak[4], aq[4];
          lda<256>(ak, sK, mt * 16, kc, lane);
          lda<256>(aq, sQ, mt * 16, kc, lane);
#pragma unroll
          for (int np = 0; np < 2; ++np) {
            uint32_t b[4];
            ldb_nk<256>(b, sK, nh * 32 + np * 16, kc * 16, lane);
            mma16816<CT>(akk[np * 2], ak, b);
            mma16816<CT>(akk[np * 2 + 1], ak, b + 2);
            mma16816<CT>(aqk[np * 2], aq, b);
            mma16816<CT>(aqk[np * 2 + 1], aq, b + 2);
          }
        }
#pragma unroll
        for (int nf = 0; nf < 4; ++nf) {
#pragma unroll
          for (int hf = 0; hf < 2; ++hf) {
            const int i = mt * 16 + qr + hf * 8;
            const int j = nh * 32 + nf * 8 + qc;
            const float gi = sG[i], bi = sB[i];
            const float d0 = i >= j ? exp2f(gi - sG[j]) : 0.f;
            const float d1 = i >= j + 1 ? exp2f(gi - sG[j + 1]) : 0.f;
            const float a0 = i > j ? bi * akk[nf][hf * 2] * d0 : 0.f;
            const float a1 = i > j + 1 ? bi * akk[nf][hf * 2 + 1] * d1 : 0.f;
            *reinterpret_cast<float2*>(sA + i * C + j) = make_float2(a0, a1);
            const float q0 = i >= j ? aqk[nf][hf * 2] * d0 : 0.f;
            const float q1 = i >= j + 1 ? aqk[nf][hf * 2 + 1] * d1 : 0.f;
            st2<CT>(sAqk, elem<128>(i, j), q0, q1);
          }
        }
      }
      __syncthreads();

      // ---- step 2: Ti = (I + A)^-1 by columns; Tu = Ti diag(beta), Tw = Ti diag(beta e^G) ----
      if (tid < C) {
        const int c = tid;
        float t[C];
#pragma unroll
        for (int i = 0; i < C; ++i) {
          float acc = i == c ? 1.f : 0.f;
#pragma unroll
          for (int j = 0; j < i; ++j) acc -= sA[i * C + j] * t[j];
          t[i] = acc;
        }
        const float bu = sB[c], bw = sB[c] * exp2f(sG[c]);
        CT* tu = reinterpret_cast<CT*>(sTu);
        CT* tw = reinterpret_cast<CT*>(sTw);
#pragma unroll
        for (int i = 0; i < C; ++i) {
          const int off = elem<128>(i, c) >> 1;
          tu[off] = from_f32<CT>(t[i] * bu);
          tw[off] = from_f32<CT>(t[i] * bw);
        }
      }
      __syncthreads();

      // ---- step 3: u = Tu v, w = Tw k  (warp: rows 16 mt, cols 64 nh) ----
      float u[8][4];
      {
        float w[8][4];
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) u[i][j] = w[i][j] = 0.f;
#pragma unroll
        for (int kc = 0; kc < C / 16; ++kc) {
          uint32_t au[4], aw[4];
          lda<128>(au, sTu, mt * 16, kc, lane);
          lda<128>(aw, sTw, mt * 16, kc, lane);
#pragma unroll
          for (int np = 0; np < 4; ++np) {
            uint32_t bv[4], bk[4];
            ldb_kn<256>(bv, sV, kc * 16, nh * 64 + np * 16, lane);
            ldb_kn<256>(bk, sK, kc * 16, nh * 64 + np * 16, lane);
            mma16816<CT>(u[np * 2], au, bv);
            mma16816<CT>(u[np * 2 + 1], au, bv + 2);
            mma16816<CT>(w[np * 2], aw, bk);
            mma16816<CT>(w[np * 2 + 1], aw, bk + 2);
          }
        }
        __syncthreads();  // sA is dead: w may overwrite it
#pragma unroll
        for (int nf = 0; nf < 8; ++nf) {
          const int col = nh * 64 + nf * 8 + qc;
          st2<CT>(sW, elem<256>(mt * 16 + qr, col), w[nf][0], w[nf][1]);
          st2<CT>(sW, elem<256>(mt * 16 + qr + 8, col), w[nf][2], w[nf][3]);
        }
      }
      __syncthreads();

      // ---- step 4: v_new = u - w S, o = e^G (q S) ----
      float o[8][4];
      {
        float ws[8][4];
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) o[i][j] = ws[i][j] = 0.f;
#pragma unroll
        for (int kc = 0; kc < KD / 16; ++kc) {
          uint32_t aw[4], aq[4];
          lda<256>(aw, sW, mt * 16, kc, lane);
          lda<256>(aq, sQ, mt * 16, kc, lane);
#pragma unroll
          for (int np = 0; np < 4; ++np) {
            uint32_t b[4];
            ldb_kn<256>(b, sS, kc * 16, nh * 64 + np * 16, lane);
            mma16816<CT>(ws[np * 2], aw, b);
            mma16816<CT>(ws[np * 2 + 1], aw, b + 2);
            mma16816<CT>(o[np * 2], aq, b);
            mma16816<CT>(o[np * 2 + 1], aq, b + 2);
          }
        }
        const int i0 = mt * 16 + qr, i1 = i0 + 8;
        const float eg0 = exp2f(sG[i0]), eg1 = exp2f(sG[i1]);
        const float gl = sG[C - 1];
        const float el0 = exp2f(gl - sG[i0]), el1 = exp2f(gl - sG[i1]);
#pragma unroll
        for (int nf = 0; nf < 8; ++nf) {
          const int col = nh * 64 + nf * 8 + qc;
          const float v00 = u[nf][0] - ws[nf][0], v01 = u[nf][1] - ws[nf][1];
          const float v10 = u[nf][2] - ws[nf][2], v11 = u[nf][3] - ws[nf][3];
          st2<CT>(sVn, elem<256>(i0, col), v00, v01);
          st2<CT>(sVn, elem<256>(i1, col), v10, v11);
          st2<CT>(sVp, elem<256>(i0, col), v00 * el0, v01 * el0);
          st2<CT>(sVp, elem<256>(i1, col), v10 * el1, v11 * el1);
          o[nf][0] *= eg0; o[nf][1] *= eg0; o[nf][2] *= eg1; o[nf][3] *= eg1;
        }
      }
      __syncthreads();

      // ---- step 5: o += Aqk v_new; store ----
      {
#pragma unroll
        for (int kc = 0; kc < C / 16; ++kc) {
          uint32_t a[4];
          lda<128>(a, sAqk, mt * 16, kc, lane);
#pragma unroll
          for (int np = 0; np < 4; ++np) {
            uint32_t b[4];
            ldb_kn<256>(b, sVn, kc * 16, nh * 64 + np * 16, lane);
            mma16816<CT>(o[np * 2], a, b);
            mma16816<CT>(o[np * 2 + 1], a, b + 2);
          }
        }
        const int i0 = mt * 16 + qr, i1 = i0 + 8;
        const float sc = p.scale;
#pragma unroll
        for (int nf = 0; nf < 8; ++nf) {
          const int col = nh * 64 + nf * 8 + qc;
          if (i0 < n)
            *reinterpret_cast<uint32_t*>(go + (c0 + i0) * p.so_t + h * p.so_h + col) =
                pack2<T>(o[nf][0] * sc, o[nf][1] * sc);
          if (i1 < n)
            *reinterpret_cast<uint32_t*>(go + (c0 + i1) * p.so_t + h * p.so_h + col) =
                pack2<T>(o[nf][2] * sc, o[nf][3] * sc);
        }
      }

      // ---- step 6: S = e^{G_last} S + k^T v'  (warp: state rows 16 warp, all 128 cols) ----
      {
        const float eL = exp2f(sG[C - 1]);
#pragma unroll
        for (int nf = 0; nf < 16; ++nf) {
          Sr[nf][0] *= eL; Sr[nf][1] *= eL; Sr[nf][2] *= eL; Sr[nf][3] *= eL;
        }
#pragma unroll
        for (int kc = 0; kc < C / 16; ++kc) {
          uint32_t a[4];
          lda_t<256>(a, sK, warp * 16, kc * 16, lane);
#pragma unroll
          for (int np = 0; np < 8; ++np) {
            uint32_t b[4];
            ldb_kn<256>(b, sVp, kc * 16, np * 16, lane);
            mma16816<CT>(Sr[np * 2], a, b);
            mma16816<CT>(Sr[np * 2 + 1], a, b + 2);
          }
        }
      }
      __syncthreads();  // every reader of sS / sK / sVp is done
#pragma unroll
      for (int nf = 0; nf < 16; ++nf) {
        const int col = nf * 8 + qc;
        st2<CT>(sS, elem<256>(warp * 16 + qr, col), Sr[nf][0], Sr[nf][1]);
        st2<CT>(sS, elem<256>(warp * 16 + qr + 8, col), Sr[nf][2], Sr[nf][3]);
      }
      // the next chunk's loads are issued after this point; sS is read only after its
      // __syncthreads, so no extra barrier is needed here
    }

    // final state
#pragma unroll
    for (int nf = 0; nf < 16; ++nf) {
      const int col = nf * 8 + qc;
      *reinterpret_cast<float2*>(gstate + (warp * 16 + qr) * p.ss_k + col) = make_float2(Sr[nf][0], Sr[nf][1]);
      *reinterpret_cast<float2*>(gstate + (warp * 16 + qr + 8) * p.ss_k + col) = make_float2(Sr[nf][2], Sr[nf][3]);
    }
    __syncthreads();  // sS of this chain is dead before the next chain writes it
  }
}

template <typename T, typename TG>
void launch_chunk(const ChunkParams& p, cudaStream_t st) {
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(gdn_chunk_kernel<T, TG>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    attr = true;
  }
  const int chains = p.n_seqs * p.hv;
  const int grid = chains < num_sms() ? chains : num_sms();
  gdn_chunk_kernel<T, TG><<<grid, kThreads, SMEM_BYTES, st>>>(p);
}

}  // namespace

int run_chunk(const char* op, const mvb_tensor* q, const mvb_tensor* k, const mvb_tensor* v, const mvb_tensor* g,
              const mvb_tensor* beta, mvb_tensor* state, const mvb_tensor* idx, const mvb_tensor* cu,
              mvb_tensor* o, float scale, int l2norm, cudaStream_t st) {
  if (cu == nullptr) MVB_FAIL(MVB_ERR_ARG, "%s: cu_seqlens is NULL", op);
  int64_t n_seqs = 0;
  int rc = check_gdn(op, q, k, v, g, beta, state, idx, cu, o, &n_seqs);
  if (rc) return rc;
  const bool fast = (q->dtype == MVB_BF16 || q->dtype == MVB_F16) && q->shape[2] == KD && v->shape[2] == VD &&
                    q->stride[2] == 1 && k->stride[2] == 1 && v->stride[2] == 1 && o->stride[2] == 1 &&
                    q->stride[0] % 8 == 0 && q->stride[1] % 8 == 0 && k->stride[0] % 8 == 0 &&
                    k->stride[1] % 8 == 0 && v->stride[0] % 8 == 0 && v->stride[1] % 8 == 0 &&
                    o->stride[0] % 2 == 0 && o->stride[1] % 2 == 0 &&
                    (reinterpret_cast<uintptr_t>(o->data) & 3) == 0 && aligned16(q->data) && aligned16(k->data) &&
                    aligned16(v->data) && state->stride[3] == 1 && state->stride[2] % 2 == 0 &&
                    (reinterpret_cast<uintptr_t>(state->data) & 7) == 0 && cu->dtype == MVB_I32 &&
                    cu->shape[0] >= 1 && (g->dtype == MVB_F32 || g->dtype == q->dtype);
  if (!fast)  // fp32 / other head sizes: token-serial recurrence (exact fp32 math)
    return run_recurrent(op, q, k, v, g, beta, state, idx, cu, o, scale, l2norm, st);
  if (n_seqs == 0 || v->shape[1] == 0) return MVB_OK;
  ChunkParams p;
  p.q = q->data; p.k = k->data; p.v = v->data; p.g = g->data; p.beta = beta->data; p.o = o->data;
  p.state = static_cast<float*>(state->data);
  p.state_idx = static_cast<const int32_t*>(idx->data);
  p.cu = static_cast<const int32_t*>(cu->data);
  p.sq_t = q->stride[0]; p.sq_h = q->stride[1]; p.sk_t = k->stride[0]; p.sk_h = k->stride[1];
  p.sv_t = v->stride[0]; p.sv_h = v->stride[1]; p.so_t = o->stride[0]; p.so_h = o->stride[1];
  p.sg_t = g->stride[0]; p.sg_h = g->stride[1]; p.sb_t = beta->stride[0]; p.sb_h = beta->stride[1];
  p.ss_n = state->stride[0]; p.ss_h = state->stride[1]; p.ss_k = state->stride[2];
  p.n_seqs = (int)n_seqs; p.hk = (int)q->shape[1]; p.hv = (int)v->shape[1]; p.l2norm = l2norm ? 1 : 0;
  p.scale = scale > 0.f ? scale : 1.0f / sqrtf((float)KD);
  const bool g32 = g->dtype == MVB_F32;
  if (q->dtype == MVB_BF16) {
    if (g32) launch_chunk<__nv_bfloat16, float>(p, st);
    else launch_chunk<__nv_bfloat16, __nv_bfloat16>(p, st);
  } else {
    if (g32) launch_chunk<__half, float>(p, st);
    else launch_chunk<__half, __half>(p, st);
  }
  MVB_CHECK_LAUNCH(op);
  return MVB_OK;
}

}  // namespace mvb

extern "C" int mvb_chunk_gated_delta_rule(const mvb_tensor* q, const mvb_tensor* k, const mvb_tensor* v,
                                          const mvb_tensor* g, const mvb_tensor* beta, mvb_tensor* recurrent_state,
                                          const mvb_tensor* recurrent_state_indices, const mvb_tensor* cu_seqlens,
                                          mvb_tensor* o, float scale, int use_qk_l2norm, void* stream) {
  return mvb::run_chunk("chunk_gated_delta_rule", q, k, v, g, beta, recurrent_state, recurrent_state_indices,
                        cu_seqlens, o, scale, use_qk_l2norm, static_cast<cudaStream_t>(stream));
}
