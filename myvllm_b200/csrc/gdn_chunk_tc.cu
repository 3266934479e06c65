// Chunked gated delta rule (prefill) on the sm_100a tensor cores: tcgen05.mma with TMEM
// accumulators, TMA-fed inputs, WY form, chunk C = 64, K = V = 128.
//
// Replaces the reference's six-launch pipeline (m/ops/gated_delta_rule/gated_delta_rule.py:44-64:
// cumsum.py -> chunk_scaled_dot_kkt.py -> solve_tril.py -> wu.py -> h.py -> o.py) with one
// persistent kernel.  A CTA walks (sequence, v-head) chains chunk by chunk; the fp32 state
// S [K, V] lives in tensor memory for the whole chain, every intermediate stays on chip, and
// HBM sees q, k, v, g, beta once, o once and the state once per chain.
//
// Per chunk (^T on a per-chunk 64-token axis; every contraction has the 128-wide feature
// dimension as the MMA M):
//   D1   = [q; k] [q; k]^T on the raw inputs    (M = N = 64 q rows + 64 k rows, K = 128);
//          its diagonal gives the q/k L2 norms, which are applied to the fp32 products:
//          Aqk = lower(scale D1[q] e^{G_i-G_j} / |q_i||k_j|),
//          A   = strict_lower(beta_i D1[k] e^{G_i-G_j} / |k_i||k_j|)
//   Ti   = (I + A)^-1                           (blocked, fp32-accurate: see solve_tril64)
//   U^T  = v^T (Ti diag(beta))^T,  W^T = k^T (Ti diag(beta e^G / |k|))^T on the raw inputs,
//          the two 64x64 factors split into 16-bit hi + lo parts (two MMAs each)
//   Vn^T = U^T - S^T W^T                         (negated-A accumulate into U^T; K = 128)
//   O^T  = S^T q'^T + Vn^T Aqk^T                 (q' = scale e^{G_i} q / |q|)
//   S    = e^{G_last} S + k'^T Vn                (k' = e^{G_last-G} k / |k|; N = 128, K = 64)
// The state-side operands (fp16 copy of S, q', k', W, Vn, Aqk) are fp16 in shared memory,
// accumulators fp32 (the final fp32 state stays within 1e-3 relative of the exact recurrence).
//
// Two warp groups pipeline consecutive chunks:
//   prep (warps 0-7): TMA loads, gates, D1, masks, triangular solve and the U/W factors for
//                     chunk c+1 -- nothing here depends on the state;
//   rec  (warps 8-11, thread = TMEM lane): q'/k', the U/W products and the W staging, then
//                     Vn, O and the state update for chunk c, the output tile and the fp16
//                     state copy for chunk c+1.
// They hand buffers over through mbarriers (normed / factors-ready / gates-ready from prep;
// MMA completions from rec).  prep publishes chunk c+1 only once the U/W products of chunk
// c are done, which keeps it at most one phase ahead on every barrier.
//
// Scheduling over the persistent grid (one CTA per SM).  With a full workspace the chains are
// balanced: laid end to end they are cut into one equal span per CTA pair, a chain cut at a
// span boundary hands its state to the next pair through recurrent_state and a flag, and the
// two CTAs of a pair (the two SMs of a TPC) run the two v-heads of one k-head side by side.
// With an 8-byte workspace whole chains go out longest sequence first through a work
// counter, without one round-robin.  Every wait is bounded; a wait that gives up sets the
// device error word and the CTA winds down.
#include <type_traits>

#include "tcgen05.cuh"
#include "tma.cuh"

namespace mvb {
namespace {

constexpr int C = 64;
constexpr int D = 128;  // K = V = 128
constexpr int kPrep = 256, kRec = 128, kThreads = kPrep + kRec;
constexpr int kBarPrep = 1, kBarRec = 2;  // named barriers
constexpr int kMaxSort = 512;

// TMEM columns (D1 is the 128 x 128 Gram matrix [q; k][q; k]^T: q columns, then k columns)
constexpr uint32_t COL_S = 0, COL_O = 128, COL_U = 192 /* two 64-column buffers */, COL_W = 320, COL_D1 = 384;
constexpr uint32_t TMEM_COLS = 512;

// shared memory (bytes from the 1024-aligned base)
constexpr uint32_t SM_QK = 0;           // raw [q; k], 2 buffers x 2 K-halves x [128 rows][128 B]
constexpr uint32_t SM_V = 65536;        // raw v, 2 halves x [64][128 B]
constexpr uint32_t SM_QP = 81920;       // q' fp16 [64 tok][128 kdim] (2 x [64][128 B])
constexpr uint32_t SM_KP = 98304;       // k' fp16 [64 tok][128 kdim]
constexpr uint32_t SM_AQK = 114688;     // Aqk fp16 [64][64]
constexpr uint32_t SM_WS = 122880;      // W^T fp16 [128 kdim][64 tok]
constexpr uint32_t SM_TF = 139264;      // Tu hi, Tu lo, Tw hi, Tw lo: 4 x [64][64] 16-bit
constexpr uint32_t SM_A = SM_TF;        //   before that: A (then M) as fp16 hi, lo planes and
constexpr uint32_t SM_T = SM_TF + 16384;  //   Ti as fp16 hi, lo planes ([64][128 B] each, swizzled)
constexpr uint32_t SM_VN = 172032;      // Vn^T fp16 [128 v][64 tok]; then the o tile [64 tok][128 v]
constexpr uint32_t SM_O = SM_VN;
constexpr uint32_t SM_S16 = 188416;     // S fp16 [128 kdim][128 v] (2 x [128][128 B])
constexpr uint32_t SM_AD = 221184;      // the 16x16 diagonal blocks of A in fp32 (4 x [16][kAdPitch])
constexpr int kAdPitch = 260;           //   block pitch in floats (bank-offset blocks)
constexpr uint32_t SM_F = 225344;       // small fp32 vectors
// Per chunk, one set by chunk parity (so that the gates and norms of chunk k+1 can be formed
// while chunk k's are still read): G (log2 units), beta, beta e^G, 1/|q|, 1/|k|,
// G - log2(1/|k|) per column.  Then the raw gates of the chunk being formed.
constexpr int F_G = 0, F_B = 64, F_BW = 128, F_QN = 192, F_KN = 256, F_GC = 320, kFSet = 384;
constexpr int F_GRAW = 2 * kFSet, F_BRAW = 2 * kFSet + 64;
constexpr uint32_t SM_PERM = SM_F + (2 * kFSet + 128) * 4;  // chain order, uint16 sequence ids
constexpr uint32_t SMEM_BYTES = SM_PERM + kMaxSort * 2 + 1024;  // + alignment slack
static_assert(SMEM_BYTES <= 232448 - 1024, "shared memory budget (with the static barriers)");
static_assert(SM_AD + 4 * kAdPitch * 4 <= SM_F, "diagonal blocks overlap the vectors");

struct Params {
  CUtensorMap tm_q, tm_k, tm_v;
  const void *g, *beta;
  void* o;
  float* state;
  const int32_t* state_idx;
  const int32_t* cu;
  int64_t so_t, so_h, sg_t, sg_h, sb_t, sb_h, ss_n, ss_h, ss_k;
  // Workspace words: [0] next chain (dynamic schedule), [1] CTAs done, [2] launch
  // generation, [3 + i] hand-off flag of CTA i (balanced schedule); or null
  int* work;
  int balanced;  // 1: balanced spans with state hand-offs (needs work[0 .. 3 + grid))
  int n_seqs, hk, hv, l2norm, g32, b32;
  float scale;
  GateDev gd;  // raw gates (a, b in the g, beta slots) when gd.alog is set
  NormDev nd;  // RMSNormGated on the output tile when nd.z is set
};

struct Bars {
  uint64_t raw_qk[2], raw_v, d1_done, mma2_done, mma_r, gready[2], r4done;
  uint64_t mma2_go, normed, mma_all, mma_all_prep;
};

// chunk record handed from prep to rec
struct Rec {
  // flags: 1 valid, 2 first chunk of a segment (load the state), 4 last chunk of a segment
  // (store the state), 8 wait for the previous CTA's hand-off first, 16 publish a hand-off
  int seq, h, c0, n, flags;
};

__device__ __forceinline__ float ldg_f(const void* p, int64_t i, bool f32, bool is_bf16) {
  if (f32) return static_cast<const float*>(p)[i];
  if (is_bf16) return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
  return __half2float(static_cast<const __half*>(p)[i]);
}

__device__ __forceinline__ void bar_sync(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }
// Barrier over a warp group that also ANDs a flag across it (uniform abort decisions).
__device__ __forceinline__ bool bar_and(int id, int n, bool v) {
  int r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.s32 p, %1, 0;\n\t"
      "bar.red.and.pred q, %2, %3, p;\n\t"
      "selp.s32 %0, 1, 0, q;\n\t}\n"
      : "=r"(r)
      : "r"((int)v), "r"(id), "r"(n)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Hand-off flags between CTAs (gpu scope): the writer's state stores are fenced before the
// release store; the reader's acquire load precedes its state loads.
__device__ __forceinline__ void st_release(int* f, int v) {
  asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(f), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire(const int* f) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
  return v;
}
// Waits (about a second at most) until *f == v; false if it gave up.
__device__ __forceinline__ bool wait_flag(const int* f, int v) {
  for (uint32_t i = 0; i < (1u << 22); ++i) {
    if (ld_acquire(f) == v) return true;
    __nanosleep(256);
  }
  return false;
}

// fp32 -> fp16 hi + lo (x ~ hi + lo to ~2^-22 relative), packed in pairs.
__device__ __forceinline__ void split2(float x0, float x1, uint32_t& hi, uint32_t& lo) {
  const __half h0 = __float2half_rn(x0), h1 = __float2half_rn(x1);
  hi = pack2<__half>(__half2float(h0), __half2float(h1));
  lo = pack2<__half>(x0 - __half2float(h0), x1 - __half2float(h1));
}

// Three independent fp32 accumulators of a 16x8 product with fp16 hi/lo operands:
// hi*hi, hi*lo and lo*hi (~fp32 accurate once summed); independent so that the three
// mma.sync of one step do not wait on each other.
struct Acc3 {
  float h[4] = {0.f, 0.f, 0.f, 0.f}, x[4] = {0.f, 0.f, 0.f, 0.f}, y[4] = {0.f, 0.f, 0.f, 0.f};
  __device__ __forceinline__ void mma(const uint32_t* ah, const uint32_t* al, const uint32_t* bh, const uint32_t* bl) {
    mma16816<__half>(h, ah, bh);
    mma16816<__half>(x, ah, bl);
    mma16816<__half>(y, al, bh);
  }
  __device__ __forceinline__ float operator[](int i) const { return h[i] + (x[i] + y[i]); }
};

// The solve's 64x64 matrices live as fp16 hi + lo planes (x ~ hi + lo, as split2 rounds it),
// each [64 rows][128 B] with the 128-byte swizzle, so that mma.sync fragments come straight
// from ldmatrix.  Element (r, c) of a plane is at sw128(r, c / 8) + 2 (c % 8).
__device__ __forceinline__ uint32_t poff(int r, int c) { return umma::sw128(r, c >> 3) + ((c & 7) << 1); }

// (x0, x1) -> columns (c, c + 1) of row r of the hi and lo planes (c even).
__device__ __forceinline__ void st_hl2(char* hi, char* lo, int r, int c, float x0, float x1) {
  uint32_t h, l;
  split2(x0, x1, h, l);
  *reinterpret_cast<uint32_t*>(hi + poff(r, c)) = h;
  *reinterpret_cast<uint32_t*>(lo + poff(r, c)) = l;
}
// 8 floats -> one 16-byte chunk of each plane.
__device__ __forceinline__ void split8(const float* x, uint4& hi, uint4& lo) {
  split2(x[0], x[1], hi.x, lo.x);
  split2(x[2], x[3], hi.y, lo.y);
  split2(x[4], x[5], hi.z, lo.z);
  split2(x[6], x[7], hi.w, lo.w);
}
// A fragment (16x16, row-major) of the block at (r0, c0).
__device__ __forceinline__ void ldsm_a(uint32_t* a, const char* plane, int r0, int c0, int lane) {
  const int mat = lane >> 3;
  ldmatrix_x4(a[0], a[1], a[2], a[3], smem_u32(plane + umma::sw128(r0 + (mat & 1) * 8 + (lane & 7), (c0 >> 3) + (mat >> 1))));
}
// B fragments of the 16 (k) x 16 (n) block at (r0, c0) stored row-major [k][n]: b[0..1] for
// columns c0..c0+7, b[2..3] for c0+8..c0+15.
__device__ __forceinline__ void ldsm_b2(uint32_t* b, const char* plane, int r0, int c0, int lane) {
  const int mat = lane >> 3;
  ldmatrix_x4_trans(b[0], b[1], b[2], b[3],
                    smem_u32(plane + umma::sw128(r0 + (mat & 1) * 8 + (lane & 7), (c0 >> 3) + (mat >> 1))));
}
// B fragment of the 16 (k) x 8 (n) block at (r0, c0).
__device__ __forceinline__ void ldsm_b1(uint32_t* b, const char* plane, int r0, int c0, int lane) {
  ldmatrix_x2_trans(b[0], b[1], smem_u32(plane + umma::sw128(r0 + ((lane >> 3) & 1) * 8 + (lane & 7), c0 >> 3)));
}

// Ti = (I + A)^-1 for the strictly lower 64x64 A; run by the 256 prep threads.  In: A as hi/lo
// planes (a_hi, a_lo) and its four diagonal 16x16 blocks in fp32 (aD).  Out: the lower part of
// Ti as hi/lo planes (t_hi, t_lo; blocks above the diagonal are left unwritten).  With
// 16x16 blocks T_ij (i >= j) and M_ik = T_ii A_ik:
//   R0  T_ii by forward substitution in fp32 (threads 0-63, one column each);
//   R1  M_ik for the six blocks below the diagonal (one warp each, written over A_ik); the
//       sub-diagonal warps go on to T_{i,i-1} = -M_{i,i-1} T_{i-1,i-1} from their registers;
//   R2  T_{j+2,j} = -(M_{j+2,j} T_jj + M_{j+2,j+1} T_{j+1,j});
//   R3  T_30 = -(M_30 T_00 + M_31 T_10 + M_32 T_20)
// (T_ij = -T_ii sum_k A_ik T_kj, the block form of forward substitution).  Products run on
// mma.sync with hi/lo operands and fp32 accumulators (hi*hi + hi*lo + lo*hi): fp32-accurate.
__device__ __forceinline__ void solve_tril64(char* a_hi, char* a_lo, const float* aD, char* t_hi, char* t_lo,
                                             int tid) {
  const int warp = tid >> 5, lane = tid & 31;
  if (tid < 64) {
    // right-looking: once x[r] is final it updates every later row, so the dependency
    // chain is 16 steps long instead of sum_r r
    const int blk = tid >> 4, base = blk * 16, c = tid & 15;
    const float* ad = aD + blk * kAdPitch;
    float x[16];
#pragma unroll
    for (int r = 0; r < 16; ++r) x[r] = r == c ? 1.f : 0.f;
#pragma unroll
    for (int r = 0; r < 16; ++r) {
#pragma unroll
      for (int r2 = r + 1; r2 < 16; ++r2) x[r2] -= ad[r2 * 16 + r] * x[r];
    }
#pragma unroll
    for (int r = 0; r < 16; ++r) {
      const __half h = __float2half_rn(x[r]);
      *reinterpret_cast<__half*>(t_hi + poff(base + r, base + c)) = h;
      *reinterpret_cast<__half*>(t_lo + poff(base + r, base + c)) = __float2half_rn(x[r] - __half2float(h));
    }
  }
  bar_sync(kBarPrep, kPrep);
  const int g = lane >> 2, q2 = (lane & 3) * 2;  // accumulator row / column pair of this lane
  if (warp < 6) {
    const int bi = warp < 3 ? warp + 1 : (warp == 5 ? 3 : warp - 1);
    const int bk = warp < 3 ? warp : (warp == 3 ? 0 : (warp == 4 ? 1 : 0));
    uint32_t ah[4], al[4], bh[4], bl[4];
    ldsm_a(ah, t_hi, bi * 16, bi * 16, lane);
    ldsm_a(al, t_lo, bi * 16, bi * 16, lane);
    ldsm_b2(bh, a_hi, bi * 16, bk * 16, lane);
    ldsm_b2(bl, a_lo, bi * 16, bk * 16, lane);
    Acc3 m0, m1;
    m0.mma(ah, al, bh, bl);
    m1.mma(ah, al, bh + 2, bl + 2);
    float m[2][4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      m[0][e] = m0[e];
      m[1][e] = m1[e];
    }
    __syncwarp();  // A_ik is read by this warp only; M_ik takes its place
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      st_hl2(a_hi, a_lo, bi * 16 + g, bk * 16 + nt * 8 + q2, m[nt][0], m[nt][1]);
      st_hl2(a_hi, a_lo, bi * 16 + g + 8, bk * 16 + nt * 8 + q2, m[nt][2], m[nt][3]);
    }
    if (warp < 3) {
      // the accumulators of the two column tiles are the A fragment of M_{i,i-1}
      split2(m[0][0], m[0][1], ah[0], al[0]);
      split2(m[0][2], m[0][3], ah[1], al[1]);
      split2(m[1][0], m[1][1], ah[2], al[2]);
      split2(m[1][2], m[1][3], ah[3], al[3]);
      ldsm_b2(bh, t_hi, bk * 16, bk * 16, lane);
      ldsm_b2(bl, t_lo, bk * 16, bk * 16, lane);
      Acc3 t0, t1;
      t0.mma(ah, al, bh, bl);
      t1.mma(ah, al, bh + 2, bl + 2);
      st_hl2(t_hi, t_lo, bi * 16 + g, bk * 16 + q2, -t0[0], -t0[1]);
      st_hl2(t_hi, t_lo, bi * 16 + g + 8, bk * 16 + q2, -t0[2], -t0[3]);
      st_hl2(t_hi, t_lo, bi * 16 + g, bk * 16 + 8 + q2, -t1[0], -t1[1]);
      st_hl2(t_hi, t_lo, bi * 16 + g + 8, bk * 16 + 8 + q2, -t1[2], -t1[3]);
    }
  }
  bar_sync(kBarPrep, kPrep);
  // R2 (warps 0-3: block row j + 2, column tile nt) and R3 (warps 4-5, after a barrier)
#pragma unroll 1
  for (int round = 2; round <= 3; ++round) {
    const bool mine = round == 2 ? warp < 4 : warp < 2;
    if (mine) {
      const int j = round == 2 ? warp >> 1 : 0, nt = warp & 1, bi = round == 2 ? j + 2 : 3;
      Acc3 acc;
      for (int kb = j; kb < bi; ++kb) {
        uint32_t ah[4], al[4], bh[2], bl[2];
        ldsm_a(ah, a_hi, bi * 16, kb * 16, lane);
        ldsm_a(al, a_lo, bi * 16, kb * 16, lane);
        ldsm_b1(bh, t_hi, kb * 16, j * 16 + nt * 8, lane);
        ldsm_b1(bl, t_lo, kb * 16, j * 16 + nt * 8, lane);
        acc.mma(ah, al, bh, bl);
      }
      st_hl2(t_hi, t_lo, bi * 16 + g, j * 16 + nt * 8 + q2, -acc[0], -acc[1]);
      st_hl2(t_hi, t_lo, bi * 16 + g + 8, j * 16 + nt * 8 + q2, -acc[2], -acc[3]);
    }
    bar_sync(kBarPrep, kPrep);
  }
}

// One chunk of a segment: a (sequence, v-head) chain, or the part of one that a CTA runs.
struct Item {
  int seq, h, c0, n, t_end;  // t_end: end token of the segment
  bool valid, first, wait, pub;
};

template <typename T, bool NORM>
__global__ void __launch_bounds__(kThreads, 1) gdn_chunk_tc_kernel(const __grid_constant__ Params p) {
  extern __shared__ __align__(1024) char smem_raw[];
  char* sm = umma::align1024(smem_raw);
  __shared__ Bars bars;
  __shared__ Rec recs[2];
  __shared__ float s_el[2];  // e^{G_last} of the chunk in each record slot
  __shared__ uint32_t tmem_slot;
  __shared__ int s_seg[5];  // next segment: seq, v-head, first chunk, end chunk, flags (1 valid, 2 wait, 4 publish)
  __shared__ int s_gen;     // launch generation (balanced schedule)
  __shared__ int s_end;  // set by prep when the work runs out

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int lane_base = (warp & 3) * 32;  // TMEM lanes this warp may access
  const int tl = tid & 127;               // TMEM lane owned by this thread
  float* sF = reinterpret_cast<float*>(sm + SM_F);
  uint16_t* sPerm = reinterpret_cast<uint16_t*>(sm + SM_PERM);
  const uint32_t sbase = smem_u32(sm);
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
  constexpr float LOG2E = 1.4426950408889634f;

  // ---- setup: chain order, barriers, TMEM ----
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
      sPerm[rank] = (uint16_t)i;
    }
  }
  if (tid == 0) {
    for (int b = 0; b < 2; ++b) {
      umma::mbar_init(&bars.raw_qk[b], 1);
      umma::mbar_init(&bars.gready[b], 1);
    }
    for (uint64_t* m : {&bars.mma2_go, &bars.normed, &bars.mma_all, &bars.mma_all_prep})
      umma::mbar_init(m, 1);
    s_end = 0;
    s_gen = p.balanced ? *reinterpret_cast<volatile int*>(p.work + 2) : 0;
    umma::mbar_init(&bars.raw_v, 1);
    umma::mbar_init(&bars.d1_done, 1);
    umma::mbar_init(&bars.mma2_done, 1);
    umma::mbar_init(&bars.mma_r, 1);
    umma::mbar_init(&bars.r4done, 1);
    umma::mbar_fence_init();
  }
  if (warp == 0) umma::tmem_alloc(&tmem_slot, TMEM_COLS);
  umma::fence_before();
  __syncthreads();
  umma::fence_after();
  const uint32_t tmem = tmem_slot;
  const int n_chains = S * p.hv;
  const uint32_t id_d1 = umma::idesc_f16(128, 128, false, false, false, kBf16);

  if (tid < kPrep) {
    // =============================================================== prep group
    // Per iteration k: mask/solve/factors of chunk k, then (while U/W(k) run on the tensor
    // core) the gates and norms of chunk k+1, then W staging and the hand-over of chunk k.
    const int wg = tid >> 7;  // column half of the TMEM tiles this thread reads
    auto seq_at = [&](int r) { return sorted ? (int)sPerm[r] : r; };
    auto nch = [&](int seq) { return (p.cu[seq + 1] - p.cu[seq] + C - 1) / C; };
    // thread 0 writes the next segment to s_seg; all prep threads then read it with seg_item
    auto put = [&](int seq, int h, int cb, int ce, int flags) {
      s_seg[0] = seq;
      s_seg[1] = h;
      s_seg[2] = cb;
      s_seg[3] = ce;
      s_seg[4] = flags;
    };
    auto seg_item = [&]() -> Item {
      Item it;
      it.valid = s_seg[4] & 1;
      it.first = true;
      it.wait = s_seg[4] & 2;
      it.pub = s_seg[4] & 4;
      if (!it.valid) return it;
      it.seq = s_seg[0];
      it.h = s_seg[1];
      const int base = p.cu[it.seq];
      it.c0 = base + s_seg[2] * C;
      it.t_end = min(p.cu[it.seq + 1], base + s_seg[3] * C);
      it.n = min(C, it.t_end - it.c0);
      return it;
    };
    // thread 0: out of work -> count this CTA out; the last CTA readies the workspace for the
    // next launch (dynamic: zero the chain counter; balanced: advance the generation)
    bool exhausted = false;
    auto count_out = [&]() {
      if (exhausted) return;
      exhausted = true;
      if (p.work && atomicAdd(p.work + 1, 1) == (int)gridDim.x - 1) {
        p.work[1] = 0;
        if (p.balanced) p.work[2] = s_gen + 1;
        else p.work[0] = 0;
      }
    };
    // Dynamic / round-robin schedule: whole chains, longest sequence first.
    int rr = 0;
    auto fetch_dynamic = [&]() {
      for (;;) {
        const int c = p.work ? atomicAdd(p.work, 1) : (int)blockIdx.x + (rr++) * (int)gridDim.x;
        if (c >= n_chains) {
          put(0, 0, 0, 0, 0);
          count_out();
          return;
        }
        const int seq = seq_at(c / p.hv), n = nch(seq);
        if (n > 0) {
          put(seq, c % p.hv, 0, n, 1);
          return;
        }
      }
    };
    // Balanced schedule (McNaughton's wrap-around rule, with the order of the two cut
    // parts chosen for a serial chain).  A unit is one sequence's v-heads 2j and 2j + 1,
    // which share a k-head; the CTA pair (2m, 2m + 1) runs its two chains side by side, cut
    // at the same places, so the two SMs of a TPC work on the same q/k tiles and the same
    // code in step (unpaired when Hv or the grid is odd).  The units laid end to end in
    // schedule order (sequences longest first) cover ntot chunks; pair m owns positions
    // [m cs, (m+1) cs), cs = max(ceil(ntot / pairs), longest chain), so the makespan is
    // about ntot / pairs chunks instead of what whole chains allow.  A unit cut at the
    // span's end (the tail cut) runs FIRST and stores its states for the next pair; a unit
    // cut at the span's start (the head cut) runs LAST and first waits for the hand-off of
    // the previous pair's CTA on the same lane.  The two parts of a unit together are at
    // most cs long, so the first is normally done before the second is reached.  Thread 0
    // only.
    const int pair = (p.hv % 2 == 0 && gridDim.x % 2 == 0) ? 2 : 1;
    const int hu = p.hv / pair, ulane = (int)blockIdx.x % pair;  // units per sequence; v-head in the unit
    int ph = 3, br = 0, bh = 0;           // phase; next whole unit (rank, unit head)
    long long bpos = 0, bend = 0;         // its start position; end of the whole chains
    int t_seq = -1, t_h = 0, t_len = 0;   // tail cut: chunks [0, t_len)
    int h_seq = -1, h_h = 0, h_off = 0;   // head cut: chunks [h_off, end)
    if (p.balanced && tid == 0) {
      long long ntot = 0;
      int maxn = 0;
      for (int sq = 0; sq < S; ++sq) {
        const int n = nch(sq);
        ntot += (long long)n * hu;
        maxn = max(maxn, n);
      }
      const long long nm = gridDim.x / pair;
      const long long cs = max((ntot + nm - 1) / nm, (long long)maxn);
      const long long A = (long long)(blockIdx.x / pair) * cs, B = min(A + cs, ntot);
      // the chain that covers position pos: rank r, head h, its start position
      auto locate = [&](long long pos, int& r, int& h, long long& start) {
        long long P = 0;
        for (r = 0; r < S; ++r) {
          const long long w = (long long)nch(seq_at(r)) * hu;
          if (P + w > pos) break;
          P += w;
        }
        const int n = nch(seq_at(r));
        h = (int)((pos - P) / n);
        start = P + (long long)h * n;
      };
      if (A < B) {
        ph = 0;
        long long sa;
        locate(A, br, bh, sa);
        bpos = sa;
        if (sa < A) {
          h_seq = seq_at(br);
          h_h = bh * pair + ulane;
          h_off = (int)(A - sa);
          bpos = sa + nch(h_seq);
          if (++bh == hu) {
            bh = 0;
            ++br;
          }
        }
        bend = B;
        if (B < ntot) {
          int rb, hb;
          long long sb;
          locate(B, rb, hb, sb);
          if (sb < B) {
            t_seq = seq_at(rb);
            t_h = hb * pair + ulane;
            t_len = (int)(B - sb);
            bend = sb;
          }
        }
      }
    }
    auto fetch_balanced = [&]() {
      if (ph == 0) {
        ph = 1;
        if (t_seq >= 0) {
          put(t_seq, t_h, 0, t_len, 1 | 4);
          return;
        }
      }
      if (ph == 1) {
        while (br < S && nch(seq_at(br)) == 0) {
          ++br;
          bh = 0;
        }
        if (br < S && bpos < bend) {
          const int sq = seq_at(br), n = nch(sq);
          put(sq, bh * pair + ulane, 0, n, 1);
          bpos += n;
          if (++bh == hu) {
            bh = 0;
            ++br;
          }
          return;
        }
        ph = 2;
      }
      if (ph == 2) {
        ph = 3;
        if (h_seq >= 0) {
          put(h_seq, h_h, h_off, nch(h_seq), 1 | 2);
          return;
        }
      }
      put(0, 0, 0, 0, 0);
      count_out();
    };
    auto fetch = [&]() {
      if (p.balanced) fetch_balanced();
      else fetch_dynamic();
    };
    // the item after `it` (fetching the next segment when `it` ends one); all prep threads call it
    auto next_item = [&](const Item& it) -> Item {
      if (!it.valid) return it;
      Item nx = it;
      if (it.c0 + C < it.t_end) {  // same segment (uniform across the group: no barrier needed)
        nx.c0 += C;
        nx.n = min(C, nx.t_end - nx.c0);
        nx.first = false;
        nx.wait = false;
        return nx;
      }
      if (tid == 0) fetch();
      bar_sync(kBarPrep, kPrep);
      nx = seg_item();
      bar_sync(kBarPrep, kPrep);  // s_seg may be rewritten by the next call
      return nx;
    };
    // loads issued / consumed (thread 0), for the drain on exit
    int qk_issued = 0, qk_used = 0, v_issued = 0, v_used = 0;
    auto issue_qk = [&](const Item& it) {
      char* dst = sm + SM_QK + (qk_issued & 1) * 32768;
      uint64_t* bar = &bars.raw_qk[qk_issued & 1];
      const int kh = it.h / (p.hv / p.hk);
      tma::expect_tx(bar, 32768);
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        tma::load_3d(dst + hh * 16384, &p.tm_q, hh * 64, kh, it.c0, bar);
        tma::load_3d(dst + hh * 16384 + 8192, &p.tm_k, hh * 64, kh, it.c0, bar);
      }
      ++qk_issued;
    };
    auto issue_v = [&](const Item& it) {
      tma::expect_tx(&bars.raw_v, 16384);
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) tma::load_3d(sm + SM_V + hh * 8192, &p.tm_v, hh * 64, it.h, it.c0, &bars.raw_v);
      ++v_issued;
    };
    float g_pre = 0.f, b_pre = 0.f;
    auto load_gates = [&](const Item& it) {
      if (!it.valid) return;
      if (tid < C) {
        g_pre = tid < it.n ? ldg_f(p.g, (int64_t)(it.c0 + tid) * p.sg_t + it.h * p.sg_h, p.g32, kBf16) : 0.f;
        if (p.gd.alog != nullptr && tid < it.n) g_pre = raw_gate_g(p.gd, g_pre, it.h);
      } else if (tid < 2 * C) {
        const int r = tid - C;
        b_pre = r < it.n ? ldg_f(p.beta, (int64_t)(it.c0 + r) * p.sb_t + it.h * p.sb_h, p.b32, kBf16) : 0.f;
        if (p.gd.alog != nullptr && r < it.n) b_pre = raw_gate_beta(b_pre, p.b32 ? MVB_F32 : (kBf16 ? MVB_BF16 : MVB_F16));
      }
    };
    bool ok = true;

    // gates of chunk kk (g_pre/b_pre hold them) -> G, beta, beta e^G; starts the loads of the
    // gates of `ahead`; publishes e^{G_last} for rec
    auto gates = [&](int kk, const Item& ahead) {
      float* fs = sF + (kk & 1) * kFSet;
      if (tid < C) sF[F_GRAW + tid] = g_pre;
      else if (tid < 2 * C) sF[F_BRAW + tid - C] = b_pre;
      bar_sync(kBarPrep, kPrep);
      load_gates(ahead);
      if (warp == 0) {
        const float g0 = sF[F_GRAW + 2 * lane], g1 = sF[F_GRAW + 2 * lane + 1];
        float incl = g0 + g1;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const float y = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= o) incl += y;
        }
        const float G0 = (incl - g1) * LOG2E, G1 = incl * LOG2E;
        const float b0 = sF[F_BRAW + 2 * lane], b1 = sF[F_BRAW + 2 * lane + 1];
        const float eg0 = exp2f(G0), eg1 = exp2f(G1);
        fs[F_G + 2 * lane] = G0;
        fs[F_G + 2 * lane + 1] = G1;
        fs[F_B + 2 * lane] = b0;
        fs[F_B + 2 * lane + 1] = b1;
        fs[F_BW + 2 * lane] = b0 * eg0;
        fs[F_BW + 2 * lane + 1] = b1 * eg1;
        const float el = __shfl_sync(0xffffffffu, eg1, 31);
        if (lane == 0) {
          s_el[kk & 1] = el;
          tma::arrive(&bars.gready[kk & 1]);
        }
      }
    };
    // raw tile of chunk kk landed -> D1 = [q; k] k^T on the tensor core (the D1 tile of chunk
    // kk-1 has been read: its mask and Aqk precede this call) -> q/k norms (and
    // G - log2(1/|k|) per k column)
    auto norms = [&](int kk) -> bool {
      bool w = umma::mbar_wait(&bars.raw_qk[kk & 1], (kk >> 1) & 1);
      if (tid == 0) qk_used = kk + 1;
      if (!(w = bar_and(kBarPrep, kPrep, w))) return false;
      if (tid == 0) {
        // D1 = [q; k] [q; k]^T: one 128-row K-major operand as both A and B
        umma::fence_after();
        const uint32_t qk_a = smem_u32(sm + SM_QK + (kk & 1) * 32768);
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
          const uint64_t d = umma::smem_desc(qk_a + (ks >> 2) * 16384 + (ks & 3) * 32, 16, 1024);
          umma::mma_f16(tmem + COL_D1, d, d, id_d1, ks > 0);
        }
        umma::commit(&bars.d1_done);
      }
      return true;
    };
    // D1 of chunk kk done -> its record, and rec may build q'/k' from here on
    auto publish_norms = [&](int kk, const Item& it) -> bool {
      bool w = umma::mbar_wait(&bars.d1_done, kk & 1);
      if (!(w = bar_and(kBarPrep, kPrep, w))) return false;
      umma::fence_after();
      // q/k norms from the Gram diagonal, D1[r][r] = |row r|^2 (rows 0-63 q, 64-127 k):
      // warps 0-3, thread = TMEM lane = row, picking column r of its warp's 32 columns
      if (tid < 128) {
        float v[32];
        umma::tmem_ld16(umma::taddr(tmem, lane_base, COL_D1 + lane_base), v);
        umma::tmem_ld16(umma::taddr(tmem, lane_base, COL_D1 + lane_base + 16), v + 16);
        umma::tmem_wait_ld();
        float ss = v[0];
#pragma unroll
        for (int j = 1; j < 32; ++j) ss = lane == j ? v[j] : ss;
        float* fs = sF + (kk & 1) * kFSet;
        const int row = tid;
        const float nf = p.l2norm ? rsqrtf(ss + 1e-6f) : 1.f;
        if (row < 64) {
          fs[F_QN + row] = nf;
        } else {
          fs[F_KN + row - 64] = nf;
          fs[F_GC + row - 64] = p.l2norm ? fs[F_G + row - 64] + 0.5f * log2f(ss + 1e-6f) : fs[F_G + row - 64];
        }
      }
      umma::fence_before();
      bar_sync(kBarPrep, kPrep);
      if (tid == 0) {
        Rec r;
        r.seq = it.seq;
        r.h = it.h;
        r.c0 = it.c0;
        r.n = it.n;
        const bool last = it.c0 + C >= it.t_end;
        r.flags = 1 | (it.first ? 2 : 0) | (last ? 4 : 0) | (it.first && it.wait ? 8 : 0) | (last && it.pub ? 16 : 0);
        recs[kk & 1] = r;
        tma::arrive(&bars.normed);
      }
      return true;
    };

    if (tid == 0) fetch();
    bar_sync(kBarPrep, kPrep);
    Item cur = seg_item();
    bar_sync(kBarPrep, kPrep);
    Item nxt = next_item(cur);
    if (tid == 0 && cur.valid) {
      tma::prefetch_map(&p.tm_q);
      tma::prefetch_map(&p.tm_k);
      tma::prefetch_map(&p.tm_v);
      issue_qk(cur);
      issue_v(cur);
      if (nxt.valid) issue_qk(nxt);
    }
    load_gates(cur);
    if (cur.valid) {
      gates(0, nxt);
      ok = norms(0) && publish_norms(0, cur);
    }

    for (int k = 0; ok; ++k) {
      if (!cur.valid) {
        // end of work: rec sees s_end on its next handshake
        if (tid == 0) {
          s_end = 1;
          tma::arrive(&bars.normed);
        }
        break;
      }

      const float* sFk = sF + (k & 1) * kFSet;  // gates and norms of chunk k
      // ---- mask and decay of the k rows: A (fp32, for the solve) ----
      // e^{G_i - G_j} / |k_j| = 2^(G_i - Gc_j) with Gc_j = G_j - log2(1/|k_j|) (log2 units);
      // masked entries may overflow before the select drops them.
      if (tl >= 64) {
        float v[32];
        umma::tmem_ld16(umma::taddr(tmem, lane_base, COL_D1 + 64 + wg * 32), v);
        umma::tmem_ld16(umma::taddr(tmem, lane_base, COL_D1 + 64 + wg * 32 + 16), v + 16);
        const int i = tl - 64;
        const float rowf = sFk[F_B + i] * sFk[F_KN + i];
        const float gi = sFk[F_G + i];
        float gc[32];
#pragma unroll
        for (int m = 0; m < 8; ++m) {
          const float4 x = *reinterpret_cast<const float4*>(sFk + F_GC + wg * 32 + 4 * m);
          gc[4 * m] = x.x; gc[4 * m + 1] = x.y; gc[4 * m + 2] = x.z; gc[4 * m + 3] = x.w;
        }
        umma::tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float e = ex2(gi - gc[j]);
          v[j] = wg * 32 + j < i ? rowf * v[j] * e : 0.f;
        }
#pragma unroll
        for (int cch = 0; cch < 4; ++cch) {
          uint4 hi, lo;
          split8(v + cch * 8, hi, lo);
          *reinterpret_cast<uint4*>(sm + SM_A + umma::sw128(i, wg * 4 + cch)) = hi;
          *reinterpret_cast<uint4*>(sm + SM_A + 8192 + umma::sw128(i, wg * 4 + cch)) = lo;
        }
        // the diagonal block of row i in fp32 for the forward substitution
        const int blk = i >> 4;
        if ((blk >> 1) == wg) {
          float* ad = reinterpret_cast<float*>(sm + SM_AD) + blk * kAdPitch + (i & 15) * 16;
          const bool up = blk & 1;  // static register indices only (no local-memory copy of v)
          float src[16];
#pragma unroll
          for (int m = 0; m < 16; ++m) src[m] = up ? v[16 + m] : v[m];
#pragma unroll
          for (int m = 0; m < 4; ++m)
            *reinterpret_cast<float4*>(ad + 4 * m) = make_float4(src[4 * m], src[4 * m + 1], src[4 * m + 2], src[4 * m + 3]);
        }
      }
      bar_sync(kBarPrep, kPrep);

      // ---- Ti = (I + A)^-1 ----
      solve_tril64(sm + SM_A, sm + SM_A + 8192, reinterpret_cast<const float*>(sm + SM_AD), sm + SM_T,
                   sm + SM_T + 8192, tid);
      if (tid == 0 && k >= 1) ok = umma::mbar_wait(&bars.r4done, (k - 1) & 1);  // Aqk buffer free
      if (!(ok = bar_and(kBarPrep, kPrep, ok))) break;

      // ---- U/W factors split hi + lo in the input type (they overwrite Ti: read all, then
      //      write); Aqk (fp16) from the q rows of D1 ----
      {
        uint4 fo[2][4];
#pragma unroll
        for (int it = 0; it < 2; ++it) {
          const int e = tid + it * kPrep;
          const int i = e >> 3, ch = e & 7;
          float uh[8], ul[8], wh[8], wl[8], th[8], tlo[8];
          unpack8<__half>(*reinterpret_cast<const uint4*>(sm + SM_T + umma::sw128(i, ch)), th);
          unpack8<__half>(*reinterpret_cast<const uint4*>(sm + SM_T + 8192 + umma::sw128(i, ch)), tlo);
#pragma unroll
          for (int jj = 0; jj < 8; ++jj) {
            const int col = ch * 8 + jj;
            const float t = i >= col ? th[jj] + tlo[jj] : 0.f;
            const float u = t * sFk[F_B + col], w = t * sFk[F_BW + col] * sFk[F_KN + col];
            uh[jj] = to_f32<T>(from_f32<T>(u));
            ul[jj] = u - uh[jj];
            wh[jj] = to_f32<T>(from_f32<T>(w));
            wl[jj] = w - wh[jj];
          }
          fo[it][0] = pack8<T>(uh);
          fo[it][1] = pack8<T>(ul);
          fo[it][2] = pack8<T>(wh);
          fo[it][3] = pack8<T>(wl);
        }
        bar_sync(kBarPrep, kPrep);
#pragma unroll
        for (int it = 0; it < 2; ++it) {
          const int e = tid + it * kPrep;
          const uint32_t off = umma::sw128(e >> 3, e & 7);
#pragma unroll
          for (int q = 0; q < 4; ++q) *reinterpret_cast<uint4*>(sm + SM_TF + q * 8192 + off) = fo[it][q];
        }
      }
      if (tl < 64) {
        float v[32];
        umma::tmem_ld16(umma::taddr(tmem, lane_base, COL_D1 + 64 + wg * 32), v);
        umma::tmem_ld16(umma::taddr(tmem, lane_base, COL_D1 + 64 + wg * 32 + 16), v + 16);
        const int i = tl;
        const float rowf = p.scale * sFk[F_QN + i];
        const float gi = sFk[F_G + i];
        float gc[32];
#pragma unroll
        for (int m = 0; m < 8; ++m) {
          const float4 x = *reinterpret_cast<const float4*>(sFk + F_GC + wg * 32 + 4 * m);
          gc[4 * m] = x.x; gc[4 * m + 1] = x.y; gc[4 * m + 2] = x.z; gc[4 * m + 3] = x.w;
        }
        umma::tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float e = ex2(gi - gc[j]);
          v[j] = wg * 32 + j <= i ? rowf * v[j] * e : 0.f;
        }
#pragma unroll
        for (int cch = 0; cch < 4; ++cch)
          *reinterpret_cast<uint4*>(sm + SM_AQK + umma::sw128(i, wg * 4 + cch)) = pack8<__half>(v + cch * 8);
      }
      umma::fence_async_smem();
      umma::fence_before();
      bar_sync(kBarPrep, kPrep);

      // ---- U^T = v^T (Tu_hi + Tu_lo)^T, W^T = k^T (Tw_hi + Tw_lo)^T (issued by rec) ----
      if (tid == 0) tma::arrive(&bars.mma2_go);

      // ---- meanwhile: gates and norms of chunk k+1 (once rec has read chunk k's) ----
      Item nxt2 = nxt;
      if (nxt.valid) {
        nxt2 = next_item(nxt);
        gates(k + 1, nxt2);
        if (!(ok = norms(k + 1))) break;
      }

      // ---- U/W(k) done: the next loads, then chunk k+1's record.  Publishing only now keeps
      //      prep one phase ahead at most: rec issued U/W(k) after taking chunk k's record and
      //      normed phase, so slot (k+1) & 1 and the next normed phase are free ----
      ok = umma::mbar_wait(&bars.mma2_done, k & 1);
      if (tid == 0) v_used = k + 1;
      if (!(ok = bar_and(kBarPrep, kPrep, ok))) break;
      if (tid == 0) {
        if (nxt.valid) issue_v(nxt);
        if (nxt2.valid && nxt.valid) issue_qk(nxt2);
      }
      if (nxt.valid && !(ok = publish_norms(k + 1, nxt))) break;
      cur = nxt;
      nxt = nxt2;
    }
    if (tid == 0) {
      if (!ok) report_device_error(1);
      // copies and D1 products still in flight (only after an abort) land before the CTA exits
      umma::commit(&bars.mma_all_prep);
      umma::mbar_wait(&bars.mma_all_prep, 0);
      for (int i = qk_used; i < qk_issued; ++i) umma::mbar_wait(&bars.raw_qk[i & 1], (i >> 1) & 1);
      for (int i = v_used; i < v_issued; ++i) umma::mbar_wait(&bars.raw_v, i & 1);
      // an aborted CTA still counts itself out so the workspace is readied for the next launch
      count_out();
    }
  } else {
    // ================================================================ rec group
    const int rt = tid - kPrep;  // == tl
    uint32_t ph = 0;             // mma_r parity
    bool ok = true;
    float* gstate = nullptr;
    T* go = static_cast<T*>(p.o);
    // Thread rt == 0 issues the tensor-core MMAs of the recurrence, in the order the pipeline
    // consumes them: U/W(k), then (after the hand-over of chunk k) Vn/O(k) and O/S-update(k).
    // prep asks for U/W with mma2_go and waits on mma2_done; rec waits on mma_r.  (prep's
    // thread 0 issues the D1 products itself: they use their own TMEM columns.)
    const uint32_t id_uw = umma::idesc_f16(128, 64, true, false, false, kBf16);
    const uint32_t id_vn = umma::idesc_f16(128, 64, true, true, true);
    const uint32_t id_sq = umma::idesc_f16(128, 64, true, false);
    const uint32_t id_o = umma::idesc_f16(128, 64, false, false);
    const uint32_t id_s = umma::idesc_f16(128, 128, true, false);
    // deferred store of the last output tile (o tile in SM_O; pend_n == 0: nothing pending)
    int pend_c0 = 0, pend_h = 0, pend_n = 0;
    // Without the layer's output norm: a plain copy of the tile.  With it, the 16 lanes of a
    // half warp that store one token row (16 x 8 columns) first form the row's RMS over the 128
    // columns by a 4-step shuffle and apply RMSNormGated to the rounded tile, as the reference
    // applies it to the op's output.
    auto store_o = [&]() {
      if constexpr (!NORM) {
        // warps 9-11 only: warp 8's lane 0 issues the U/W products meanwhile
        for (int e = rt - 32; e < C * 16; e += kRec - 32) {
          if (e < 0) break;
          const int i = e >> 4, c16 = e & 15;
          if (i < pend_n) {
            const uint4 val = *reinterpret_cast<const uint4*>(sm + SM_O + (c16 >> 3) * 8192 + umma::sw128(i, c16 & 7));
            *reinterpret_cast<uint4*>(go + (int64_t)(pend_c0 + i) * p.so_t + (int64_t)pend_h * p.so_h + c16 * 8) = val;
          }
        }
      } else {
        // this thread's columns are fixed (c16 = rt & 15): their norm weights, then the z rows
        // of all its tokens in flight at once, then the rows
        const int c16 = rt & 15;
        float nw8[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) nw8[j] = load_scalar(p.nd.w, c16 * 8 + j, p.nd.w_dt);
        uint4 zr[C * 16 / kRec];
#pragma unroll
        for (int it = 0; it < C * 16 / kRec; ++it) {
          const int i = (rt + it * kRec) >> 4;
          zr[it] = i < pend_n ? *reinterpret_cast<const uint4*>(static_cast<const T*>(p.nd.z) +
                                                                 (int64_t)(pend_c0 + i) * p.nd.z_t +
                                                                 (int64_t)pend_h * p.nd.z_h + c16 * 8)
                              : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int it = 0; it < C * 16 / kRec; ++it) {  // uniform trip count: every lane shuffles
          const int i = (rt + it * kRec) >> 4;
          const bool live = i < pend_n;
          float f[8], zf[8];
          unpack8<T>(live ? *reinterpret_cast<const uint4*>(sm + SM_O + (c16 >> 3) * 8192 + umma::sw128(i, c16 & 7))
                          : make_uint4(0, 0, 0, 0),
                     f);
          float ss = 0.f;
#pragma unroll
          for (int j = 0; j < 8; ++j) ss += f[j] * f[j];
#pragma unroll
          for (int off = 1; off < 16; off <<= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
          if (live) {
            const float r = rsqrtf(ss / (float)D + p.nd.eps);
            unpack8<T>(zr[it], zf);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              // silu(z) = z sigmoid(z) = 0.5 z (1 + tanh(z / 2)): one MUFU op
              const float hz = 0.5f * zf[j];
              float th;
              asm("tanh.approx.f32 %0, %1;" : "=f"(th) : "f"(hz));
              f[j] = f[j] * r * nw8[j] * fmaf(hz, th, hz);
            }
            *reinterpret_cast<uint4*>(go + (int64_t)(pend_c0 + i) * p.so_t + (int64_t)pend_h * p.so_h + c16 * 8) =
                pack8<T>(f);
          }
        }
      }
      pend_n = 0;
    };
    for (int k = 0; ok; ++k) {
      const int b = k & 1;
      // ---- q' = scale e^{G_i} q / |q| and k' = e^{G_last - G_i} k / |k| (fp16) for chunk k,
      //      from the raw tile while prep masks and solves it; thread = row of [q; k] ----
      ok = umma::mbar_wait(&bars.normed, k & 1);
      if (!(ok = bar_and(kBarRec, kRec, ok))) break;
      if (*reinterpret_cast<volatile int*>(&s_end)) break;
      {
        const char* qk = sm + SM_QK + b * 32768;
        const int i = rt & 63;
        float sc;
        const float* sFk = sF + b * kFSet;
        if (rt < 64) sc = p.scale * exp2f(sFk[F_G + i]) * sFk[F_QN + i];
        else sc = i < recs[b].n ? exp2f(sFk[F_G + C - 1] - sFk[F_G + i]) * sFk[F_KN + i] : 0.f;
        char* dst = sm + (rt < 64 ? SM_QP : SM_KP);
        // all 16 loads first: the stores below go to other buffers, but the compiler cannot
        // prove it and would otherwise order every load after the previous store
        uint4 raw[16];
#pragma unroll
        for (int hh = 0; hh < 2; ++hh)
#pragma unroll
          for (int c = 0; c < 8; ++c) raw[hh * 8 + c] = *reinterpret_cast<const uint4*>(qk + hh * 16384 + umma::sw128(rt, c));
#pragma unroll
        for (int hh = 0; hh < 2; ++hh)
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            float f[8];
            unpack8<T>(raw[hh * 8 + c], f);
#pragma unroll
            for (int j = 0; j < 8; ++j) f[j] *= sc;
            *reinterpret_cast<uint4*>(dst + hh * 8192 + umma::sw128(i, c)) = pack8<__half>(f);
          }
      }
      umma::fence_async_smem();
      bar_sync(kBarRec, kRec);

      // ---- U^T = v^T (Tu_hi + Tu_lo)^T, W^T = k^T (Tw_hi + Tw_lo)^T once prep has the factors ----
      if (rt == 0) {
        ok = umma::mbar_wait(&bars.mma2_go, k & 1) && umma::mbar_wait(&bars.raw_v, k & 1);
        if (ok) {
          umma::fence_after();
          const uint32_t qk_a = sbase + SM_QK + b * 32768, tf = sbase + SM_TF;
#pragma unroll
          for (int ks = 0; ks < C / 16; ++ks) {
            const uint64_t a_v = umma::desc_mnmajor(sbase + SM_V, 8192, ks);
            const uint64_t a_k = umma::desc_mnmajor(qk_a + 8192, 16384, ks);
            umma::mma_f16(tmem + COL_U + b * 64, a_v, umma::smem_desc(tf + ks * 32, 16, 1024), id_uw, ks > 0);
            umma::mma_f16(tmem + COL_U + b * 64, a_v, umma::smem_desc(tf + 8192 + ks * 32, 16, 1024), id_uw, true);
            umma::mma_f16(tmem + COL_W, a_k, umma::smem_desc(tf + 16384 + ks * 32, 16, 1024), id_uw, ks > 0);
            umma::mma_f16(tmem + COL_W, a_k, umma::smem_desc(tf + 24576 + ks * 32, 16, 1024), id_uw, true);
          }
          umma::commit(&bars.mma2_done);
        }
      }
      store_o();  // the previous chunk's output tile, while thread 0 issues the MMAs above
      if (!(ok = bar_and(kBarRec, kRec, ok))) break;

      // ---- U/W done: stage W^T [kdim][tok] (fp16, MN-major B operand of the Vn MMA) ----
      ok = umma::mbar_wait(&bars.mma2_done, k & 1);
      if (!(ok = bar_and(kBarRec, kRec, ok))) break;
      umma::fence_after();
      {
        float v[64];
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) umma::tmem_ld16(umma::taddr(tmem, lane_base, COL_W + q4 * 16), v + q4 * 16);
        umma::tmem_wait_ld();
#pragma unroll
        for (int cch = 0; cch < 8; ++cch)
          *reinterpret_cast<uint4*>(sm + SM_WS + umma::sw128(tl, cch)) = pack8<__half>(v + cch * 8);
      }
      const Rec rec = recs[b];
      umma::fence_async_smem();
      umma::fence_before();
      bar_sync(kBarRec, kRec);

      // ---- segment start: state -> TMEM (pre-scaled by e^{G_last}) and its fp16 copy; a
      //      head cut first waits for the previous CTA to hand the state over ----
      if (rec.flags & 2) {
        if (rec.flags & 8) {
          // the unit's previous part ran on the same lane of the previous CTA pair
          const int pair = (p.hv % 2 == 0 && gridDim.x % 2 == 0) ? 2 : 1;
          if (rt == 0) ok = wait_flag(p.work + 3 + blockIdx.x - pair, s_gen + 1);
          if (!(ok = bar_and(kBarRec, kRec, ok))) break;
        }
        gstate = p.state + (int64_t)p.state_idx[rec.seq] * p.ss_n + (int64_t)rec.h * p.ss_h;
        const float el = s_el[b];
        const float* srow = gstate + (int64_t)tl * p.ss_k;
#pragma unroll 2
        for (int cc = 0; cc < D; cc += 16) {
          float v[16];
#pragma unroll
          for (int j = 0; j < 16; j += 4) {
            const float4 x = __ldcg(reinterpret_cast<const float4*>(srow + cc + j));  // L2: may be a hand-off
            v[j] = x.x; v[j + 1] = x.y; v[j + 2] = x.z; v[j + 3] = x.w;
          }
#pragma unroll
          for (int j = 0; j < 16; j += 8) {
            const int col = cc + j;
            *reinterpret_cast<uint4*>(sm + SM_S16 + (col >> 6) * 16384 + umma::sw128(tl, (col >> 3) & 7)) =
                pack8<__half>(v + j);
          }
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] *= el;
          umma::tmem_st16(umma::taddr(tmem, lane_base, COL_S + cc), v);
        }
        umma::tmem_wait_st();
        umma::fence_async_smem();
        umma::fence_before();
        bar_sync(kBarRec, kRec);
      }

      // ---- Vn^T = U^T - S^T W^T,  O^T = S^T q'^T ----
      if (rt == 0) {
        umma::fence_after();
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
          const uint64_t a_s = umma::desc_mnmajor(sbase + SM_S16, 16384, ks);
          umma::mma_f16(tmem + COL_U + b * 64, a_s, umma::desc_mnmajor(sbase + SM_WS, 8192, ks), id_vn, true);
          umma::mma_f16(tmem + COL_O, a_s, umma::desc_kmajor(sbase + SM_QP, 64, ks), id_sq, ks > 0);
        }
        umma::commit(&bars.mma_r);
      }
      ok = umma::mbar_wait(&bars.mma_r, ph);
      ph ^= 1;
      if (!(ok = bar_and(kBarRec, kRec, ok))) break;
      umma::fence_after();

      // ---- stage Vn^T [v][tok] (fp16, K-major) ----
      {
        float v[64];
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) umma::tmem_ld16(umma::taddr(tmem, lane_base, COL_U + b * 64 + q4 * 16), v + q4 * 16);
        umma::tmem_wait_ld();
#pragma unroll
        for (int cch = 0; cch < 8; ++cch)
          *reinterpret_cast<uint4*>(sm + SM_VN + umma::sw128(tl, cch)) = pack8<__half>(v + cch * 8);
      }
      umma::fence_async_smem();
      umma::fence_before();
      bar_sync(kBarRec, kRec);

      // ---- O^T += Vn^T Aqk^T,  S += k'^T Vn ----
      if (rt == 0) {
        umma::fence_after();
#pragma unroll
        for (int ks = 0; ks < C / 16; ++ks) {
          const uint64_t vn = umma::desc_kmajor(sbase + SM_VN, 128, ks);
          umma::mma_f16(tmem + COL_O, vn, umma::desc_kmajor(sbase + SM_AQK, 64, ks), id_o, true);
          umma::mma_f16(tmem + COL_S, umma::desc_mnmajor(sbase + SM_KP, 8192, ks), vn, id_s, true);
        }
        umma::commit(&bars.r4done);
        umma::commit(&bars.mma_r);
      }
      ok = umma::mbar_wait(&bars.mma_r, ph);
      ph ^= 1;
      if (!(ok = bar_and(kBarRec, kRec, ok))) break;
      umma::fence_after();

      // ---- epilogue: o tile; fp16 copy of S and S e^{G_last} for the next chunk, or the
      //      final state ----
      T* ot = reinterpret_cast<T*>(sm + SM_O);  // [64 tok][128 v], 2 v-halves of [64][128 B]
      {
        float v[64];
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) umma::tmem_ld16(umma::taddr(tmem, lane_base, COL_O + q4 * 16), v + q4 * 16);
        umma::tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 64; ++j) ot[umma::elem_off(j, tl, 8192) >> 1] = from_f32<T>(v[j]);
      }
      if (rec.flags & 4) {
        float* srow = gstate + (int64_t)tl * p.ss_k;
#pragma unroll 2
        for (int cc = 0; cc < D; cc += 16) {
          float v[16];
          umma::tmem_ld16(umma::taddr(tmem, lane_base, COL_S + cc), v);
          umma::tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 16; j += 4)
            *reinterpret_cast<float4*>(srow + cc + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
        }
        if (rec.flags & 16) __threadfence();  // the hand-off: state stores before the flag
      } else {
        const int nb = (k + 1) & 1;
        ok = umma::mbar_wait(&bars.gready[nb], ((k + 1) >> 1) & 1);
        const float el = s_el[nb];
#pragma unroll 1
        for (int cc = 0; cc < D; cc += 64) {
          float v[64];
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) umma::tmem_ld16(umma::taddr(tmem, lane_base, COL_S + cc + q4 * 16), v + q4 * 16);
          umma::tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 64; j += 8) {
            const int col = cc + j;
            *reinterpret_cast<uint4*>(sm + SM_S16 + (col >> 6) * 16384 + umma::sw128(tl, (col >> 3) & 7)) =
                pack8<__half>(v + j);
          }
#pragma unroll
          for (int j = 0; j < 64; ++j) v[j] *= el;
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) umma::tmem_st16(umma::taddr(tmem, lane_base, COL_S + cc + q4 * 16), v + q4 * 16);
        }
        umma::tmem_wait_st();
      }
      umma::fence_async_smem();
      umma::fence_before();
      if (!(ok = bar_and(kBarRec, kRec, ok))) break;
      if ((rec.flags & 16) && rt == 0) st_release(p.work + 3 + blockIdx.x, s_gen + 1);
      // the tile goes to HBM in the next chunk's U/W window (SM_O is next written by its Vn
      // staging, which follows the hand-over of that chunk)
      pend_c0 = rec.c0;
      pend_h = rec.h;
      pend_n = rec.n;
      if constexpr (NORM) {  // the z rows of this tile into L2 now, for the store a chunk later
        if (rt < pend_n)
          asm volatile("cp.async.bulk.prefetch.L2.global [%0], 256;" ::"l"(static_cast<const T*>(p.nd.z) +
                                                                         (int64_t)(pend_c0 + rt) * p.nd.z_t +
                                                                         (int64_t)pend_h * p.nd.z_h)
                       : "memory");
      }
    }
    if (ok) store_o();
    if (rt == 0) {
      if (!ok) report_device_error(1);
      // every MMA issued so far completes before TMEM is freed
      umma::commit(&bars.mma_all);
      umma::mbar_wait(&bars.mma_all, 0);
    }
  }

  umma::fence_before();
  __syncthreads();
  if (warp == 0) {
    umma::fence_after();
    umma::tmem_dealloc(tmem, TMEM_COLS);
  }
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

// Workspace of the balanced schedule for a grid of `grid` CTAs: the dynamic chain counter,
// the done counter, the launch generation and one hand-off flag per CTA (int32 words).
size_t chunk_gdn_workspace_bytes(int grid) { return sizeof(int) * (3 + (size_t)grid); }

// Returns -1 when the TMA descriptors cannot be built (the caller then runs the token-serial
// kernel), else an MVB status.
int launch_chunk_tc(const mvb_tensor* q, const mvb_tensor* k, const mvb_tensor* v, const mvb_tensor* g,
                    const mvb_tensor* beta, mvb_tensor* state, const mvb_tensor* idx, const mvb_tensor* cu,
                    mvb_tensor* o, float scale, int l2norm, int64_t n_seqs, int* work, size_t work_bytes,
                    const GateDev& gd, cudaStream_t st, const NormDev& nd) {
  Params p;
  memset(&p, 0, sizeof(p));
  const int64_t T_tok = q->shape[0];
  const cuuint32_t box[3] = {64, 1, (cuuint32_t)C};
  auto map3 = [&](CUtensorMap* m, const mvb_tensor* t) {
    const cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)t->shape[1], (cuuint64_t)T_tok};
    const cuuint64_t str[2] = {(cuuint64_t)t->stride[1] * 2, (cuuint64_t)t->stride[0] * 2};
    return tma::encode(m, q->dtype, 3, t->data, dims, str, box);
  };
  if (!map3(&p.tm_q, q) || !map3(&p.tm_k, k) || !map3(&p.tm_v, v)) return -1;
  p.work = work;
  p.g = g->data; p.beta = beta->data; p.o = o->data;
  p.state = static_cast<float*>(state->data);
  p.state_idx = static_cast<const int32_t*>(idx->data);
  p.cu = static_cast<const int32_t*>(cu->data);
  p.so_t = o->stride[0]; p.so_h = o->stride[1];
  p.sg_t = g->stride[0]; p.sg_h = g->stride[1]; p.sb_t = beta->stride[0]; p.sb_h = beta->stride[1];
  p.ss_n = state->stride[0]; p.ss_h = state->stride[1]; p.ss_k = state->stride[2];
  p.n_seqs = (int)n_seqs; p.hk = (int)q->shape[1]; p.hv = (int)v->shape[1];
  p.l2norm = l2norm ? 1 : 0; p.g32 = g->dtype == MVB_F32; p.b32 = beta->dtype == MVB_F32;
  p.scale = scale > 0.f ? scale : 1.0f / sqrtf((float)D);
  p.gd = gd;
  p.nd = nd;
  const int chains = (int)(n_seqs * p.hv);
  const int grid = chains < num_sms() ? chains : num_sms();
  // the balanced schedule has CTAs wait for each other's hand-offs: a cooperative launch
  // guarantees that the whole grid (one CTA per SM) is resident at once
  p.balanced = work != nullptr && work_bytes >= chunk_gdn_workspace_bytes(grid) ? 1 : 0;
  const bool norm = nd.z != nullptr;
  // the four kernels share one function-pointer type: each keeps its own attribute mask
  static unsigned long long mask_bf = 0, mask_bf_norm = 0, mask_h = 0, mask_h_norm = 0;
  auto go = [&](auto kernel, unsigned long long& attr_mask) -> cudaError_t {
    ensure_smem_attr(kernel, SMEM_BYTES, attr_mask);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = SMEM_BYTES;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = p.balanced ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, p);
  };
  auto launch = [&]() -> cudaError_t {
    if (q->dtype == MVB_BF16)
      return norm ? go(gdn_chunk_tc_kernel<__nv_bfloat16, true>, mask_bf_norm)
                  : go(gdn_chunk_tc_kernel<__nv_bfloat16, false>, mask_bf);
    return norm ? go(gdn_chunk_tc_kernel<__half, true>, mask_h_norm) : go(gdn_chunk_tc_kernel<__half, false>, mask_h);
  };
  cudaError_t e = launch();
  if (e == cudaErrorCooperativeLaunchTooLarge && p.balanced) {
    // fewer SMs usable than the grid (e.g. an MPS thread limit): whole chains through the
    // dynamic counter need no co-residency (work[0] and work[1] are the same words)
    (void)cudaGetLastError();
    p.balanced = 0;
    e = launch();
  }
  if (e != cudaSuccess) MVB_FAIL(MVB_ERR_CUDA, "chunk_gated_delta_rule: launch failed: %s", cudaGetErrorString(e));
  MVB_CHECK_LAUNCH("chunk_gated_delta_rule");
  return MVB_OK;
}

}  // namespace mvb
