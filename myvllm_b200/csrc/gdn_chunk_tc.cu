// Chunked gated delta rule (prefill) on the sm_100a tensor cores: tcgen05.mma with TMEM
// accumulators, WY form, chunk C = 64, K = V = 128.
//
// Replaces the reference's six-launch pipeline (m/ops/gated_delta_rule/gated_delta_rule.py:44-64:
// cumsum.py -> chunk_scaled_dot_kkt.py -> solve_tril.py -> wu.py -> h.py -> o.py) with one
// persistent kernel.  A CTA walks one (sequence, v-head) chain chunk by chunk; the fp32 state
// S [K, V] lives in tensor memory for the whole chain, every intermediate stays on chip, and
// HBM sees q, k, v, g, beta once, o once and the state once per chain.
//
// Every contraction is written with the 128-wide feature dimension as the MMA M (the only
// M=128 cta_group::1 shape), i.e. transposed where needed (^T on a per-chunk 64-token axis):
//   D1   = [q; k] k^T                 (M = 64 q rows + 64 k rows, N = 64, K = 128)
//          -> Aqk = lower(D1[q] * e^{G_i-G_j}),  A = strict_lower(beta_i D1[k] e^{G_i-G_j})
//   Ti   = (I + A)^-1                 (blocked: 16x16 diagonal blocks by fp32 forward
//                                      substitution, off-diagonal blocks by mma.sync with
//                                      fp16 hi/lo operand splitting, ~fp32 accurate)
//   U^T  = v^T (Ti diag(beta))^T      W^T = k^T (Ti diag(beta e^G))^T          (N = 64, K = 64)
//   Vn^T = U^T - S^T W^T              (negated-A accumulate into U^T; K = 128)
//   O1^T = S^T q^T,   O2^T = Vn^T Aqk^T,   o = scale (e^{G_i} O1 + O2)
//   S    = e^{G_last} S + k'^T Vn     (k' = e^{G_last - G} k; N = 128, K = 64)
// Operands are fp16 in shared memory (bf16 inputs convert exactly; see the precision note
// in run_chunk), staged in the 128-byte-swizzle layouts of tcgen05.cuh; accumulators fp32.
//
// Per chunk the CTA (256 threads = 2 warpgroups; thread t of a warpgroup owns TMEM lane t,
// the two warpgroups split columns) runs: convert tiles (+ q/k L2 norm) and prefetch the next
// chunk with cp.async -> MMA D1, O1 -> masks/decay -> solve -> MMA U, W -> stage W ->
// MMA Vn -> stage Vn, scale S -> MMA O2, S-update -> epilogue (o, fp16 copy of S).
// Chains are handed out longest sequence first over a persistent grid (one CTA per SM):
// dynamically through a work counter when the caller supplies one (CTAs that finish early
// take the next chain; the last CTA to run dry zeroes the counter for the next launch),
// else round-robin.
#include <type_traits>

#include "tcgen05.cuh"

namespace mvb {

int check_gdn(const char* op, const mvb_tensor* q, const mvb_tensor* k, const mvb_tensor* v, const mvb_tensor* g,
              const mvb_tensor* beta, const mvb_tensor* state, const mvb_tensor* idx, const mvb_tensor* cu,
              const mvb_tensor* o, int64_t* n_seqs_out);
int run_recurrent(const char* op, const mvb_tensor* q, const mvb_tensor* k, const mvb_tensor* v,
                  const mvb_tensor* g, const mvb_tensor* beta, mvb_tensor* state, const mvb_tensor* idx,
                  const mvb_tensor* cu, mvb_tensor* o, float scale, int l2norm, cudaStream_t st);

namespace {

constexpr int C = 64;
constexpr int D = 128;  // K = V = 128
constexpr int kThreads = 256;
constexpr int kMaxSort = 512;

// TMEM columns
constexpr uint32_t COL_S = 0, COL_D1 = 128, COL_U = 192, COL_W = 256, COL_O1 = 320, COL_O2 = 384;
constexpr uint32_t TMEM_COLS = 512;

// shared memory (bytes from the 1024-aligned base)
constexpr uint32_t SM_QK = 0;          // [q;k] fp16, 2 K-halves x [128][128 B]
constexpr uint32_t SM_V = 32768;       // v fp16, 2 halves x [64][128 B]
constexpr uint32_t SM_KP = 49152;      // k' fp16
constexpr uint32_t SM_S = 65536;       // S fp16, 2 v-halves x [128][128 B]
constexpr uint32_t SM_W = 98304;       // w fp16 [64 tokens][128 kdim]
constexpr uint32_t SM_VN = 114688;     // v_new fp16 [64 tokens][128 v]
constexpr uint32_t SM_TU = 131072;     // Tu fp16 [64][64]
constexpr uint32_t SM_TW = 139264;     // Tw fp16 [64][64]
constexpr uint32_t SM_AQK = 147456;    // Aqk fp16 [64][64]
constexpr uint32_t SM_A = 155648;      // A fp32 [64][64], column index XOR-swizzled by row
constexpr uint32_t SM_T = SM_W;        // Ti fp32 [64][64] (same swizzle), aliases w (dead then)
constexpr uint32_t SM_X = SM_VN;       // per-warp 16x16 fp32 scratch of the solve, aliases v_new
constexpr uint32_t SM_STG = 172032;    // staging (raw inputs): q, k, v, each 2 halves x [64][128 B]
constexpr uint32_t SM_G = 221184;      // G2 [64] f32
constexpr uint32_t SM_B = SM_G + 256;  // beta [64] f32
constexpr uint32_t SM_BW = SM_B + 256; // beta e^G [64] f32
constexpr uint32_t SM_AL = SM_BW + 256; // e^{g_t} [64] f32 (per-token decay)
constexpr uint32_t SM_EG = SM_AL + 256; // e^{G_t} [64] f32
constexpr uint32_t SM_O = SM_W;         // o tile [64][128] of the epilogue (w is dead by then)
constexpr uint32_t SM_PERM = SM_EG + 256;
constexpr uint32_t SMEM_BYTES = SM_PERM + kMaxSort * 4 + 1024;  // + alignment slack

struct Params {
  const void *q, *k, *v, *g, *beta;
  void* o;
  float* state;
  const int32_t* state_idx;
  const int32_t* cu;
  int64_t sq_t, sq_h, sk_t, sk_h, sv_t, sv_h, so_t, so_h, sg_t, sg_h, sb_t, sb_h;
  int64_t ss_n, ss_h, ss_k;
  int* work;  // [next chain, CTAs done] or null
  int n_seqs, hk, hv, l2norm, g32, b32;
  float scale;
};

__device__ __forceinline__ float ldg_f(const void* p, int64_t i, bool f32, bool is_bf16) {
  if (f32) return static_cast<const float*>(p)[i];
  if (is_bf16) return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
  return __half2float(static_cast<const __half*>(p)[i]);
}

// fp32 [64][64] matrices of the solve: element (i, j) at i * 64 + (j ^ (i & 31)).
__device__ __forceinline__ int fidx(int i, int j) { return i * 64 + (j ^ (i & 31)); }

// fp32 -> fp16 hi + lo (x ~ hi + lo to ~2^-22 relative), packed in pairs.
__device__ __forceinline__ void split2(float x0, float x1, uint32_t& hi, uint32_t& lo) {
  const __half h0 = __float2half_rn(x0), h1 = __float2half_rn(x1);
  hi = pack2<__half>(__half2float(h0), __half2float(h1));
  lo = pack2<__half>(x0 - __half2float(h0), x1 - __half2float(h1));
}

// A fragment (16x16) of block (bi, bj) of a swizzled fp32 [64][64] matrix, split hi/lo.
__device__ __forceinline__ void frag_a_split(uint32_t* ah, uint32_t* al, const float* M, int bi, int bj, int lane) {
  const int r = bi * 16 + (lane >> 2), c = bj * 16 + (lane & 3) * 2;
  split2(M[fidx(r, c)], M[fidx(r, c + 1)], ah[0], al[0]);
  split2(M[fidx(r + 8, c)], M[fidx(r + 8, c + 1)], ah[1], al[1]);
  split2(M[fidx(r, c + 8)], M[fidx(r, c + 9)], ah[2], al[2]);
  split2(M[fidx(r + 8, c + 8)], M[fidx(r + 8, c + 9)], ah[3], al[3]);
}

// acc (16x8) += A B with fp16 hi/lo operands: hi*hi + hi*lo + lo*hi (~fp32 accurate).
__device__ __forceinline__ void mma3(float* acc, const uint32_t* ah, const uint32_t* al, const uint32_t* bh,
                                     const uint32_t* bl) {
  mma16816<__half>(acc, ah, bh);
  mma16816<__half>(acc, ah, bl);
  mma16816<__half>(acc, al, bh);
}

// Ti = (I + A)^-1 for the strictly lower 64x64 A in sA; result (lower part) in sT.
// Diagonal 16x16 blocks by right-looking forward substitution (threads 0-63), then for each
// block diagonal L = 1, 2, 3 every (block (i, j = i - L), 8-column tile) pair is one warp:
//   X = sum_{k=j}^{i-1} A_ik T_kj[:, tile],   T_ij[:, tile] = -T_ii X
// with the products on mma.sync (fp16 hi/lo splitting, fp32 accumulate).
__device__ __forceinline__ void solve_tril64(const float* sA, float* sT, float* sX, int tid) {
  const int warp = tid >> 5, lane = tid & 31;
  if (tid < 64) {
    // right-looking: once x[r] is final it updates every later row, so the dependency
    // chain is 16 steps long instead of sum_r r
    const int base = (tid >> 4) * 16, c = tid & 15;
    float x[16];
#pragma unroll
    for (int r = 0; r < 16; ++r) x[r] = r == c ? 1.f : 0.f;
#pragma unroll
    for (int r = 0; r < 16; ++r) {
#pragma unroll
      for (int r2 = r + 1; r2 < 16; ++r2) x[r2] -= sA[fidx(base + r2, base + r)] * x[r];
    }
#pragma unroll
    for (int r = 0; r < 16; ++r) sT[fidx(base + r, base + c)] = x[r];
  }
  __syncthreads();
  const int r = lane >> 2, c2 = (lane & 3) * 2;
#pragma unroll 1
  for (int lvl = 1; lvl < 4; ++lvl) {
    if (warp < 2 * (4 - lvl)) {
      const int bj = warp >> 1, bi = bj + lvl, nt = warp & 1;
      float X[4] = {0.f, 0.f, 0.f, 0.f};
      for (int kb = bj; kb < bi; ++kb) {
        uint32_t ah[4], al[4], bh[2], bl[2];
        frag_a_split(ah, al, sA, bi, kb, lane);
        const int k = kb * 16 + c2, n = bj * 16 + nt * 8 + r;
        split2(sT[fidx(k, n)], sT[fidx(k + 1, n)], bh[0], bl[0]);
        split2(sT[fidx(k + 8, n)], sT[fidx(k + 9, n)], bh[1], bl[1]);
        mma3(X, ah, al, bh, bl);
      }
      // X (16 x 8, accumulator layout) -> per-warp scratch -> B-operand layout
      float* xs = sX + warp * 128;  // [16][8]
      xs[r * 8 + c2] = X[0]; xs[r * 8 + c2 + 1] = X[1];
      xs[(r + 8) * 8 + c2] = X[2]; xs[(r + 8) * 8 + c2 + 1] = X[3];
      __syncwarp();
      uint32_t ah[4], al[4], bh[2], bl[2];
      frag_a_split(ah, al, sT, bi, bi, lane);
      split2(xs[c2 * 8 + r], xs[(c2 + 1) * 8 + r], bh[0], bl[0]);
      split2(xs[(c2 + 8) * 8 + r], xs[(c2 + 9) * 8 + r], bh[1], bl[1]);
      float Y[4] = {0.f, 0.f, 0.f, 0.f};
      mma3(Y, ah, al, bh, bl);
      const int rr = bi * 16 + r, cc = bj * 16 + nt * 8 + c2;
      sT[fidx(rr, cc)] = -Y[0]; sT[fidx(rr, cc + 1)] = -Y[1];
      sT[fidx(rr + 8, cc)] = -Y[2]; sT[fidx(rr + 8, cc + 1)] = -Y[3];
    }
    __syncthreads();
  }
}

// One work item = (chain, chunk).  Chain j of this CTA is blockIdx.x + j * gridDim.x in the
// longest-first order.
struct Item {
  int seq, h, c0, n, t_end;
  bool valid;
};

template <typename T>
__global__ void __launch_bounds__(kThreads, 1) gdn_chunk_tc_kernel(Params p) {
  extern __shared__ __align__(1024) char smem_raw[];
  char* sm = umma::align1024(smem_raw);
  __shared__ uint64_t mbar;
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;
  __shared__ float s_graw[C], s_braw[C];
  __shared__ int s_chain;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int wg = warp >> 2;          // warpgroup: splits TMEM columns
  const int tl = tid & 127;          // TMEM lane owned by this thread
  const int lane_base = (warp & 3) * 32;
  float* sG = reinterpret_cast<float*>(sm + SM_G);
  float* sB = reinterpret_cast<float*>(sm + SM_B);
  float* sBW = reinterpret_cast<float*>(sm + SM_BW);
  float* sAL = reinterpret_cast<float*>(sm + SM_AL);
  float* sEG = reinterpret_cast<float*>(sm + SM_EG);
  float* sT = reinterpret_cast<float*>(sm + SM_T);
  float* sX = reinterpret_cast<float*>(sm + SM_X);
  int* sPerm = reinterpret_cast<int*>(sm + SM_PERM);
  float* sA = reinterpret_cast<float*>(sm + SM_A);
  const uint32_t sbase = smem_u32(sm);
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr float LOG2E = 1.4426950408889634f;

  // ---- setup: chain order, barrier, TMEM ----
  const int S = p.n_seqs;
  const bool sorted = S <= kMaxSort;
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
  if (tid == 0) {
    umma::mbar_init(&mbar, 1);
    umma::mbar_fence_init();
    abort_flag = 0;
  }
  if (warp == 0) umma::tmem_alloc(&tmem_slot, TMEM_COLS);
  umma::fence_before();
  __syncthreads();
  umma::fence_after();
  const uint32_t tmem = tmem_slot;
  uint32_t phase = 0;

  const T* gq = static_cast<const T*>(p.q);
  const T* gk = static_cast<const T*>(p.k);
  const T* gv = static_cast<const T*>(p.v);
  T* go = static_cast<T*>(p.o);
  const int n_chains = S * p.hv;

  auto chain_item = [&](int chain) -> Item {
    Item it;
    it.valid = chain < n_chains;
    if (!it.valid) return it;
    it.seq = sorted ? sPerm[chain / p.hv] : chain / p.hv;
    it.h = chain % p.hv;
    it.c0 = p.cu[it.seq];
    it.t_end = p.cu[it.seq + 1];
    it.n = min(C, it.t_end - it.c0);
    return it;
  };
  // Thread 0 only: the next non-empty chain for this CTA (>= n_chains when none is left).
  int rr = 0;
  bool exhausted = false;
  auto fetch = [&]() -> int {
    for (;;) {
      const int c = p.work ? atomicAdd(p.work, 1) : (int)blockIdx.x + (rr++) * (int)gridDim.x;
      if (c >= n_chains) {
        exhausted = true;
        if (p.work && atomicAdd(p.work + 1, 1) == (int)gridDim.x - 1) {
          p.work[0] = 0;
          p.work[1] = 0;
        }
        return c;
      }
      if (chain_item(c).n > 0) return c;
    }
  };
  // Prefetch raw q/k/v of an item into staging (cp.async, zero rows >= n); g/beta into regs.
  float g_pre = 0.f, b_pre = 0.f;
  auto prefetch = [&](const Item& it) {
    if (!it.valid) return;
    const int kh = it.h / (p.hv / p.hk);
    for (int i = tid; i < C * 16; i += kThreads) {
      const int r = i >> 4, c = i & 15;
      const bool ok = r < it.n;
      const int t = ok ? it.c0 + r : it.c0;
      const uint32_t off = (c >> 3) * 8192 + umma::sw128(r, c & 7);
      cp_async16(sm + SM_STG + off, gq + t * p.sq_t + kh * p.sq_h + c * 8, ok);
      cp_async16(sm + SM_STG + 16384 + off, gk + t * p.sk_t + kh * p.sk_h + c * 8, ok);
      cp_async16(sm + SM_STG + 32768 + off, gv + t * p.sv_t + it.h * p.sv_h + c * 8, ok);
    }
    cp_async_commit();
    if (tid < C) {
      g_pre = tid < it.n ? ldg_f(p.g, (int64_t)(it.c0 + tid) * p.sg_t + it.h * p.sg_h, p.g32, kBf16) : 0.f;
    } else if (tid < 2 * C) {
      const int r = tid - C;
      b_pre = r < it.n ? ldg_f(p.beta, (int64_t)(it.c0 + r) * p.sb_t + it.h * p.sb_h, p.b32, kBf16) : 0.f;
    }
  };
  // wait for the MMAs committed so far; all threads take part
  auto mma_wait = [&]() -> bool {
    if (!umma::mbar_wait(&mbar, phase)) {
      abort_flag = 1;
      report_device_error(1);
    }
    phase ^= 1;
    umma::fence_after();
    return true;
  };

  if (tid == 0) s_chain = fetch();
  __syncthreads();
  int chain = s_chain;
  Item cur = chain_item(chain);
  prefetch(cur);
  bool chain_start = true;

  float* gstate = nullptr;
  while (cur.valid) {
    const int h = cur.h, c0 = cur.c0, n = cur.n;
    const bool last_chunk = c0 + C >= cur.t_end;
    if (chain_start) gstate = p.state + (int64_t)p.state_idx[cur.seq] * p.ss_n + (int64_t)h * p.ss_h;

    // ---- chain start: state -> TMEM (fp32) and SM_S (fp16) ----
    if (chain_start) {
      const float* srow = gstate + (int64_t)tl * p.ss_k + wg * 64;
#pragma unroll
      for (int cc = 0; cc < 64; cc += 16) {
        float v[16];
#pragma unroll
        for (int j = 0; j < 16; j += 4) {
          const float4 x = *reinterpret_cast<const float4*>(srow + cc + j);
          v[j] = x.x; v[j + 1] = x.y; v[j + 2] = x.z; v[j + 3] = x.w;
        }
        umma::tmem_st16(umma::taddr(tmem, lane_base, COL_S + wg * 64 + cc), v);
        // fp16 copy: row tl (kdim), columns wg*64 + cc .. +16 -> two 16-byte chunks
#pragma unroll
        for (int j = 0; j < 16; j += 8) {
          const int col = wg * 64 + cc + j;
          *reinterpret_cast<uint4*>(sm + SM_S + (col >> 6) * 16384 + umma::sw128(tl, (col >> 3) & 7)) =
              pack8<__half>(v + j);
        }
      }
      umma::tmem_wait_st();
    }

    // ---- A: chunk landed; G, beta ----
    cp_async_wait<0>();
    if (tid < C) s_graw[tid] = g_pre;
    else if (tid < 2 * C) s_braw[tid - C] = b_pre;
    if (last_chunk && tid == 0) s_chain = fetch();
    __syncthreads();
    if (warp == 0) {
      const float g0 = s_graw[2 * lane], g1 = s_graw[2 * lane + 1];
      float incl = g0 + g1;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      sG[2 * lane] = (incl - g1) * LOG2E;
      sG[2 * lane + 1] = incl * LOG2E;
      sB[2 * lane] = s_braw[2 * lane];
      sB[2 * lane + 1] = s_braw[2 * lane + 1];
      const float eg0 = exp2f((incl - g1) * LOG2E), eg1 = exp2f(incl * LOG2E);
      sEG[2 * lane] = eg0;
      sEG[2 * lane + 1] = eg1;
      sBW[2 * lane] = s_braw[2 * lane] * eg0;
      sBW[2 * lane + 1] = s_braw[2 * lane + 1] * eg1;
      sAL[2 * lane] = exp2f(g0 * LOG2E);
      sAL[2 * lane + 1] = exp2f(g1 * LOG2E);
    }
    __syncthreads();

    // ---- B: convert staging -> fp16 operands (q, k L2-normalised; k' = e^{G_last-G} k) ----
    {
      const int r = tid >> 2, qq = tid & 3;  // row, quarter of the 128 columns
      const float gl = sG[C - 1];
      const float kscale = exp2f(gl - sG[r]);
#pragma unroll
      for (int m = 0; m < 2; ++m) {
        float f[4][8];
        float ss = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int c = qq * 4 + i;
          const uint32_t off = (c >> 3) * 8192 + umma::sw128(r, c & 7);
          unpack8<T>(*reinterpret_cast<const uint4*>(sm + SM_STG + m * 16384 + off), f[i]);
#pragma unroll
          for (int j = 0; j < 8; ++j) ss += f[i][j] * f[i][j];
        }
        float sc = 1.f;
        if (p.l2norm) {
          ss += __shfl_xor_sync(0xffffffffu, ss, 1);
          ss += __shfl_xor_sync(0xffffffffu, ss, 2);
          sc = rsqrtf(ss + 1e-6f);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int c = qq * 4 + i;
          float y[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) y[j] = f[i][j] * sc;
          // [q;k]: q rows 0-63, k rows 64-127 of each 16 KB K-half
          *reinterpret_cast<uint4*>(sm + SM_QK + (c >> 3) * 16384 + umma::sw128(r + m * 64, c & 7)) =
              pack8<__half>(y);
          if (m == 1) {
#pragma unroll
            for (int j = 0; j < 8; ++j) y[j] *= kscale;
            *reinterpret_cast<uint4*>(sm + SM_KP + (c >> 3) * 8192 + umma::sw128(r, c & 7)) = pack8<__half>(y);
          }
        }
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int c = qq * 4 + i;
        const uint32_t off = (c >> 3) * 8192 + umma::sw128(r, c & 7);
        float f[8];
        unpack8<T>(*reinterpret_cast<const uint4*>(sm + SM_STG + 32768 + off), f);
        *reinterpret_cast<uint4*>(sm + SM_V + off) = pack8<__half>(f);
      }
    }
    umma::fence_async_smem();
    umma::fence_before();
    __syncthreads();
    umma::fence_after();
    // staging is free: prefetch the next item while this one computes
    Item nxt = cur;
    int next_chain = chain;
    if (last_chunk) {
      next_chain = s_chain;
      nxt = chain_item(next_chain);
    } else {
      nxt.c0 += C;
      nxt.n = min(C, nxt.t_end - nxt.c0);
    }
    prefetch(nxt);

    // ---- MMA 1: D1 = [q;k] k^T, O1^T = S^T q^T ----
    if (tid == 0) {
      const uint32_t id_d1 = umma::idesc_f16(128, 64, false, false);
      const uint32_t id_o1 = umma::idesc_f16(128, 64, true, false);
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks) {
        const uint32_t koff = (ks >> 2) * 16384 + (ks & 3) * 32;
        const uint64_t a_qk = umma::smem_desc(sbase + SM_QK + koff, 16, 1024);
        const uint64_t b_k = umma::smem_desc(sbase + SM_QK + 8192 + koff, 16, 1024);
        umma::mma_f16(tmem + COL_D1, a_qk, b_k, id_d1, ks > 0);
        const uint64_t a_st = umma::desc_mnmajor(sbase + SM_S, 16384, ks);
        const uint64_t b_q = umma::smem_desc(sbase + SM_QK + koff, 16, 1024);
        umma::mma_f16(tmem + COL_O1, a_st, b_q, id_o1, ks > 0);
      }
      umma::commit(&mbar);
    }
    mma_wait();

    // ---- masks and decay: Aqk (fp16, K-major B operand) and A (fp32 for the solve) ----
    // d(i, j) = e^{G_i - G_j} along a row by the recurrence d(i, j-1) = d(i, j) e^{g_j},
    // restarted at d(i, i) = 1: one multiply per entry instead of an exponential.
    {
      float v[32];
      umma::tmem_ld16(umma::taddr(tmem, lane_base, COL_D1 + wg * 32), v);
      umma::tmem_ld16(umma::taddr(tmem, lane_base, COL_D1 + wg * 32 + 16), v + 16);
      umma::tmem_wait_ld();
      const int i = tl & 63;
      const bool qrow = tl < 64;
      const float bi = qrow ? 1.f : sB[i];
      const int jhi = wg * 32 + 31;
      float d = i > jhi ? exp2f(sG[i] - sG[jhi]) : 1.f;  // e^{G_i - G_jhi} for rows below the range
#pragma unroll
      for (int j = 31; j >= 0; --j) {
        const int jj = wg * 32 + j;
        if (jj == i) d = 1.f;
        const bool keep = qrow ? jj <= i : jj < i;
        v[j] = keep ? bi * v[j] * d : 0.f;
        d *= sAL[jj];
      }
      if (qrow) {
#pragma unroll
        for (int cch = 0; cch < 4; ++cch)
          *reinterpret_cast<uint4*>(sm + SM_AQK + umma::sw128(i, wg * 4 + cch)) = pack8<__half>(v + cch * 8);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) sA[fidx(i, wg * 32 + j)] = v[j];
      }
    }
    __syncthreads();

    // ---- solve Ti = (I + A)^-1; Tu = Ti diag(beta), Tw = Ti diag(beta e^G) (fp16, K-major) ----
    solve_tril64(sA, sT, sX, tid);
    for (int e = tid; e < C * 8; e += kThreads) {
      const int i = e >> 3, ch = e & 7;
      float u[8], w[8];
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) {
        const int col = ch * 8 + jj;
        const float t = i >= col ? sT[fidx(i, col)] : 0.f;
        u[jj] = t * sB[col];
        w[jj] = t * sBW[col];
      }
      *reinterpret_cast<uint4*>(sm + SM_TU + umma::sw128(i, ch)) = pack8<__half>(u);
      *reinterpret_cast<uint4*>(sm + SM_TW + umma::sw128(i, ch)) = pack8<__half>(w);
    }
    umma::fence_async_smem();
    __syncthreads();

    // ---- MMA 2: U^T = v^T Tu^T, W^T = k^T Tw^T ----
    if (tid == 0) {
      umma::fence_after();
      const uint32_t id = umma::idesc_f16(128, 64, true, false);
#pragma unroll
      for (int ks = 0; ks < C / 16; ++ks) {
        const uint64_t b_tu = umma::smem_desc(sbase + SM_TU + ks * 32, 16, 1024);
        const uint64_t b_tw = umma::smem_desc(sbase + SM_TW + ks * 32, 16, 1024);
        umma::mma_f16(tmem + COL_U, umma::desc_mnmajor(sbase + SM_V, 8192, ks), b_tu, id, ks > 0);
        umma::mma_f16(tmem + COL_W, umma::desc_mnmajor(sbase + SM_QK + 8192, 16384, ks), b_tw, id, ks > 0);
      }
      umma::commit(&mbar);
    }
    mma_wait();

    // ---- stage w (tokens x kdim, K-major B operand) ----
    {
      float v[32];
      umma::tmem_ld16(umma::taddr(tmem, lane_base, COL_W + wg * 32), v);
      umma::tmem_ld16(umma::taddr(tmem, lane_base, COL_W + wg * 32 + 16), v + 16);
      umma::tmem_wait_ld();
      __half* w = reinterpret_cast<__half*>(sm + SM_W);
      const int d = tl;  // kdim
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int i = wg * 32 + j;  // token
        w[umma::elem_off(i, d, 8192) >> 1] = __float2half_rn(v[j]);
      }
    }
    umma::fence_async_smem();
    umma::fence_before();
    __syncthreads();

    // ---- MMA 3: Vn^T = U^T - S^T W^T ----
    if (tid == 0) {
      umma::fence_after();
      const uint32_t id = umma::idesc_f16(128, 64, true, false, true);
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks) {
        const uint64_t b_w = umma::smem_desc(sbase + SM_W + (ks >> 2) * 8192 + (ks & 3) * 32, 16, 1024);
        umma::mma_f16(tmem + COL_U, umma::desc_mnmajor(sbase + SM_S, 16384, ks), b_w, id, true);
      }
      umma::commit(&mbar);
    }
    mma_wait();

    // ---- stage v_new (tokens x v), scale S by e^{G_last} in TMEM ----
    {
      float v[32];
      umma::tmem_ld16(umma::taddr(tmem, lane_base, COL_U + wg * 32), v);
      umma::tmem_ld16(umma::taddr(tmem, lane_base, COL_U + wg * 32 + 16), v + 16);
      umma::tmem_wait_ld();
      __half* vn = reinterpret_cast<__half*>(sm + SM_VN);
      const int vc = tl;  // v column
#pragma unroll
      for (int j = 0; j < 32; ++j) vn[umma::elem_off(wg * 32 + j, vc, 8192) >> 1] = __float2half_rn(v[j]);
      const float eL = exp2f(sG[C - 1]);
#pragma unroll
      for (int cc = 0; cc < 64; cc += 16) {
        float s16[16];
        const uint32_t a = umma::taddr(tmem, lane_base, COL_S + wg * 64 + cc);
        umma::tmem_ld16(a, s16);
        umma::tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 16; ++j) s16[j] *= eL;
        umma::tmem_st16(a, s16);
      }
      umma::tmem_wait_st();
    }
    umma::fence_async_smem();
    umma::fence_before();
    __syncthreads();

    // ---- MMA 4: O2^T = Vn^T Aqk^T, S += k'^T Vn ----
    if (tid == 0) {
      umma::fence_after();
      const uint32_t id_o2 = umma::idesc_f16(128, 64, true, false);
      const uint32_t id_s = umma::idesc_f16(128, 128, true, true);
#pragma unroll
      for (int ks = 0; ks < C / 16; ++ks) {
        const uint64_t a_vn = umma::desc_mnmajor(sbase + SM_VN, 8192, ks);
        const uint64_t b_aqk = umma::smem_desc(sbase + SM_AQK + ks * 32, 16, 1024);
        umma::mma_f16(tmem + COL_O2, a_vn, b_aqk, id_o2, ks > 0);
        umma::mma_f16(tmem + COL_S, umma::desc_mnmajor(sbase + SM_KP, 8192, ks), a_vn, id_s, true);
      }
      umma::commit(&mbar);
    }
    mma_wait();

    // ---- epilogue: o = scale (e^{G_i} O1 + O2) via a shared tile (16-byte global stores);
    //      fp16 copy of S (and the final fp32 state) ----
    {
      float o1[32], o2[32];
      umma::tmem_ld16(umma::taddr(tmem, lane_base, COL_O1 + wg * 32), o1);
      umma::tmem_ld16(umma::taddr(tmem, lane_base, COL_O1 + wg * 32 + 16), o1 + 16);
      umma::tmem_ld16(umma::taddr(tmem, lane_base, COL_O2 + wg * 32), o2);
      umma::tmem_ld16(umma::taddr(tmem, lane_base, COL_O2 + wg * 32 + 16), o2 + 16);
      umma::tmem_wait_ld();
      T* ot = reinterpret_cast<T*>(sm + SM_O);  // [64 tokens][128 v], 2 v-halves of [64][128 B]
      const int vc = tl;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int i = wg * 32 + j;
        ot[umma::elem_off(i, vc, 8192) >> 1] = from_f32<T>(p.scale * (sEG[i] * o1[j] + o2[j]));
      }
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        float s32[32];
        umma::tmem_ld16(umma::taddr(tmem, lane_base, COL_S + wg * 64 + half * 32), s32);
        umma::tmem_ld16(umma::taddr(tmem, lane_base, COL_S + wg * 64 + half * 32 + 16), s32 + 16);
        umma::tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 32; j += 8) {
          const int col = wg * 64 + half * 32 + j;
          *reinterpret_cast<uint4*>(sm + SM_S + (col >> 6) * 16384 + umma::sw128(tl, (col >> 3) & 7)) =
              pack8<__half>(s32 + j);
        }
        if (last_chunk) {
          float* srow = gstate + (int64_t)tl * p.ss_k + wg * 64 + half * 32;
#pragma unroll
          for (int j = 0; j < 32; j += 4)
            *reinterpret_cast<float4*>(srow + j) = make_float4(s32[j], s32[j + 1], s32[j + 2], s32[j + 3]);
        }
      }
      __syncthreads();
      // o tile -> global, 16 bytes per access
      for (int e = tid; e < C * 16; e += kThreads) {
        const int i = e >> 4, c16 = e & 15;
        if (i < n) {
          const uint4 val = *reinterpret_cast<const uint4*>(sm + SM_O + (c16 >> 3) * 8192 + umma::sw128(i, c16 & 7));
          *reinterpret_cast<uint4*>(go + (int64_t)(c0 + i) * p.so_t + (int64_t)h * p.so_h + c16 * 8) = val;
        }
      }
    }
    umma::fence_async_smem();
    umma::fence_before();
    __syncthreads();
    umma::fence_after();
    if (abort_flag) break;

    chain_start = last_chunk;
    chain = next_chain;
    cur = nxt;
  }

  // an aborted CTA still counts itself out so the work counter is zeroed for the next launch
  if (tid == 0 && p.work && !exhausted && atomicAdd(p.work + 1, 1) == (int)gridDim.x - 1) {
    p.work[0] = 0;
    p.work[1] = 0;
  }
  cp_async_wait<0>();
  umma::fence_before();
  __syncthreads();
  if (warp == 0) umma::tmem_dealloc(tmem, TMEM_COLS);
}

}  // namespace

// Shape/stride gate for the tensor-core path.
bool chunk_tc_supported(const mvb_tensor* q, const mvb_tensor* k, const mvb_tensor* v, const mvb_tensor* g,
                        const mvb_tensor* beta, const mvb_tensor* state, const mvb_tensor* o) {
  return (q->dtype == MVB_BF16 || q->dtype == MVB_F16) && q->shape[2] == D && v->shape[2] == D &&
         q->stride[2] == 1 && k->stride[2] == 1 && v->stride[2] == 1 && o->stride[2] == 1 &&
         o->stride[0] % 8 == 0 && o->stride[1] % 8 == 0 && aligned16(o->data) && q->stride[0] % 8 == 0 &&
         q->stride[1] % 8 == 0 && k->stride[0] % 8 == 0 && k->stride[1] % 8 == 0 && v->stride[0] % 8 == 0 &&
         v->stride[1] % 8 == 0 && aligned16(q->data) && aligned16(k->data) && aligned16(v->data) &&
         state->stride[3] == 1 && state->stride[2] % 4 == 0 && state->stride[1] % 4 == 0 &&
         state->stride[0] % 4 == 0 && aligned16(state->data) && (g->dtype == MVB_F32 || g->dtype == q->dtype) &&
         (beta->dtype == MVB_F32 || beta->dtype == q->dtype);
}

int launch_chunk_tc(const mvb_tensor* q, const mvb_tensor* k, const mvb_tensor* v, const mvb_tensor* g,
                    const mvb_tensor* beta, mvb_tensor* state, const mvb_tensor* idx, const mvb_tensor* cu,
                    mvb_tensor* o, float scale, int l2norm, int64_t n_seqs, int* work, cudaStream_t st) {
  Params p;
  p.work = work;
  p.q = q->data; p.k = k->data; p.v = v->data; p.g = g->data; p.beta = beta->data; p.o = o->data;
  p.state = static_cast<float*>(state->data);
  p.state_idx = static_cast<const int32_t*>(idx->data);
  p.cu = static_cast<const int32_t*>(cu->data);
  p.sq_t = q->stride[0]; p.sq_h = q->stride[1]; p.sk_t = k->stride[0]; p.sk_h = k->stride[1];
  p.sv_t = v->stride[0]; p.sv_h = v->stride[1]; p.so_t = o->stride[0]; p.so_h = o->stride[1];
  p.sg_t = g->stride[0]; p.sg_h = g->stride[1]; p.sb_t = beta->stride[0]; p.sb_h = beta->stride[1];
  p.ss_n = state->stride[0]; p.ss_h = state->stride[1]; p.ss_k = state->stride[2];
  p.n_seqs = (int)n_seqs; p.hk = (int)q->shape[1]; p.hv = (int)v->shape[1];
  p.l2norm = l2norm ? 1 : 0; p.g32 = g->dtype == MVB_F32; p.b32 = beta->dtype == MVB_F32;
  p.scale = scale > 0.f ? scale : 1.0f / sqrtf((float)D);
  const int chains = (int)(n_seqs * p.hv);
  const int grid = chains < num_sms() ? chains : num_sms();
  if (q->dtype == MVB_BF16) {
    static unsigned long long attr_mask = 0;
    ensure_smem_attr(gdn_chunk_tc_kernel<__nv_bfloat16>, SMEM_BYTES, attr_mask);
    gdn_chunk_tc_kernel<__nv_bfloat16><<<grid, kThreads, SMEM_BYTES, st>>>(p);
  } else {
    static unsigned long long attr_mask = 0;
    ensure_smem_attr(gdn_chunk_tc_kernel<__half>, SMEM_BYTES, attr_mask);
    gdn_chunk_tc_kernel<__half><<<grid, kThreads, SMEM_BYTES, st>>>(p);
  }
  MVB_CHECK_LAUNCH("chunk_gated_delta_rule");
  return MVB_OK;
}

}  // namespace mvb
