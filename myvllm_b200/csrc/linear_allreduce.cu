// Row-parallel output projection fused with its all-reduce: out = sum over ranks of
// x_r W_r^T, the o_proj / out_proj of a tensor-parallel attention layer followed by the
// dist.all_reduce of RowParallelLinear.forward (reference m/layers/linear.py:159-164), in one
// kernel per rank over NVLink peer memory.  Decode-size inputs: M <= 128 tokens.
//
// Every launch runs kCtas = 128 CTAs.  CTA c owns output columns [64 t, 64 t + 64) of tile
// t = c / S and the K blocks of split s = c % S (S = 128 / tiles; 64-wide K blocks):
//   1. GEMM on the tensor core: x [M, K] and W [N, K] tiles arrive by TMA (this GPU's memory
//      only, no multicast) in a 4-stage ring; one thread issues tcgen05.mma (M = 128 rows,
//      N = 64, fp32 accumulator in TMEM; x rows past M are zero-filled by TMA);
//   2. the 128 x 64 fp32 partial goes to this rank's IPC buffer (slot e & 1 of call e), and
//      a release store of e into flags[slot][rank][c] of every rank (this one included)
//      publishes it;
//   3. CTA c then reduces rows [s 128/S, (s+1) 128/S) of tile t: it waits (acquire, bounded)
//      for the flags of all world x S contributors of the tile, reads their partials with
//      plain loads (peers' through NVLink), adds them in (rank, split) order -- so every rank
//      gets the same bits -- and writes the bf16 output rows < M.
// Two slots alternate as in the one-shot all-reduce (allreduce.cu): a rank starts call e+2
// only after its call e+1 finished, in which every contributor of its tiles had published
// call e+1, which they do only after their call e finished reading; all 128 CTAs run on every
// call, so the per-CTA call counters stay equal.  A wait that gives up sets the device error
// word and the CTA writes zeros for its rows.
//
// Buffer layout (mvb_linear_allreduce_buffer_bytes):
//   [0, 8192)       flags   uint32 [2 slots][8 ranks][128 CTAs]
//   [8192, 8704)    epochs  uint32 [128 CTAs]
//   [16384, ...)    partials fp32, 2 slots x 128 CTAs x [128 rows][64 cols]
#include <type_traits>

#include "tcgen05.cuh"
#include "tma.cuh"

namespace mvb {
namespace {

using namespace umma;

constexpr int kCtas = 128;
constexpr int kThreads = 128;
constexpr int kMaxRanks = MVB_AR_MAX_RANKS;
constexpr int BM = 128, BN = 64, BK = 64, NS = 4;
constexpr uint32_t A_BYTES = BM * BK * 2, B_BYTES = BN * BK * 2, STAGE = A_BYTES + B_BYTES;
constexpr uint32_t SMEM = NS * STAGE + 1024;
constexpr size_t kFlagsOff = 0, kEpochOff = 8192, kDataOff = 16384;
constexpr size_t kTileBytes = (size_t)BM * BN * 4;
constexpr size_t kSlotBytes = (size_t)kCtas * kTileBytes;
constexpr uint32_t kSpinLimit = 1u << 22;
constexpr int kErrLinearAr = 6;

struct LaParams {
  CUtensorMap tm_x, tm_w;
  char* bufs[kMaxRanks];
  void* out;
  int64_t so;
  int M, N, world, rank, splits, kb_per_split;
};

struct LaBars {
  uint64_t full[NS], empty[NS], done;
  uint32_t tmem;
  int fail;
  uint32_t epoch;
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void load_2d(void* dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(smem_u32(dst)),
      "l"(map), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1) linear_allreduce_kernel(const __grid_constant__ LaParams p) {
  extern __shared__ __align__(1024) char smem_raw[];
  char* sm = align1024(smem_raw);
  __shared__ LaBars bars;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int c = blockIdx.x, t = c / p.splits, s = c % p.splits;
  const int kb0 = s * p.kb_per_split, nkb = p.kb_per_split;
  char* mine = p.bufs[p.rank];
  uint32_t* epochs = reinterpret_cast<uint32_t*>(mine + kEpochOff);
  constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;

  if (tid == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&bars.full[i], 1);
      mbar_init(&bars.empty[i], 1);
    }
    mbar_init(&bars.done, 1);
    mbar_fence_init();
    bars.fail = 0;
    bars.epoch = epochs[c] + 1;
  }
  if (warp == 0) tmem_alloc(&bars.tmem, BN);
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = bars.tmem, e = bars.epoch;
  const int slot = e & 1;

  // ---- 1. the partial GEMM tile ----
  int issued = 0;
  if (warp == 0 && lane == 0) {  // TMA producer
    tma::prefetch_map(&p.tm_x);
    tma::prefetch_map(&p.tm_w);
    bool ok = true;
    for (int i = 0; i < nkb && ok; ++i) {
      const int st = i % NS;
      if (i >= NS && !(ok = mbar_wait(&bars.empty[st], ((i / NS) & 1) ^ 1))) break;
      char* a = sm + st * STAGE;
      tma::expect_tx(&bars.full[st], STAGE);
      load_2d(a, &p.tm_x, (kb0 + i) * BK, 0, &bars.full[st]);
      load_2d(a + A_BYTES, &p.tm_w, (kb0 + i) * BK, t * BN, &bars.full[st]);
      issued = i + 1;
    }
    if (!ok) atomicExch(&bars.fail, 1);
  } else if (warp == 1 && lane == 0) {  // MMA issuer
    const uint32_t id = idesc_f16(BM, BN, false, false, false, kBf16);
    bool ok = true;
    for (int i = 0; i < nkb && ok; ++i) {
      const int st = i % NS;
      if (!(ok = mbar_wait(&bars.full[st], (i / NS) & 1))) break;
      fence_after();
      const uint32_t a = smem_u32(sm + st * STAGE), b = a + A_BYTES;
#pragma unroll
      for (int ks = 0; ks < BK / 16; ++ks) mma_f16(tmem, desc_kmajor(a, BM, ks), desc_kmajor(b, BN, ks), id, i > 0 || ks > 0);
      commit(&bars.empty[st]);
    }
    commit(&bars.done);  // also after a failure: every issued MMA completes before TMEM is freed
    if (!ok) atomicExch(&bars.fail, 1);
  }
  __syncwarp();
  // every thread = one row of the tile (TMEM lane)
  bool ok = mbar_wait(&bars.done, 0);
  fence_after();
  float* part = reinterpret_cast<float*>(mine + kDataOff + slot * kSlotBytes + (size_t)c * kTileBytes);
  {
    float v[BN];
#pragma unroll
    for (int q = 0; q < BN / 16; ++q) tmem_ld16(taddr(tmem, warp * 32, q * 16), v + q * 16);
    tmem_wait_ld();
    float4* row = reinterpret_cast<float4*>(part + (size_t)tid * BN);
#pragma unroll
    for (int q = 0; q < BN / 4; ++q) row[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
  }
  fence_before();
  if (!ok) atomicExch(&bars.fail, 1);
  if (warp == 0 && lane == 0) {  // copies still in flight (only after a failed wait) land first
    for (int i = issued > NS ? issued - NS : 0; i < issued; ++i) mbar_wait(&bars.full[i % NS], (i / NS) & 1);
  }
  __syncthreads();

  // ---- 2. publish this partial to every rank ----
  if (tid < p.world) {
    __threadfence_system();
    st_release_sys(reinterpret_cast<uint32_t*>(p.bufs[tid] + kFlagsOff) + (slot * kMaxRanks + p.rank) * kCtas + c, e);
  }
  // ---- 3. wait for the tile's world x S contributors, then reduce this CTA's rows ----
  const int n_contrib = p.world * p.splits;
  if (tid < n_contrib) {
    const int r = tid / p.splits, c2 = t * p.splits + tid % p.splits;
    const uint32_t* f = reinterpret_cast<const uint32_t*>(mine + kFlagsOff) + (slot * kMaxRanks + r) * kCtas + c2;
    uint32_t it = 0;
    while (ld_acquire_sys(f) != e) {
      if (++it == kSpinLimit) {
        atomicExch(&bars.fail, 1);
        break;
      }
      __nanosleep(64);
    }
  }
  __syncthreads();
  const bool failed = bars.fail != 0;
  if (failed && tid == 0) report_device_error(kErrLinearAr);
  const int rows = BM / p.splits, r0 = s * rows;
  T* out = static_cast<T*>(p.out);
  for (int idx = tid; idx < rows * (BN / 4); idx += kThreads) {
    const int row = r0 + idx / (BN / 4), q = idx % (BN / 4);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    if (!failed) {
      for (int r = 0; r < p.world; ++r) {
        const char* base = p.bufs[r] + kDataOff + slot * kSlotBytes;
        for (int s2 = 0; s2 < p.splits; ++s2) {
          const float4 x = __ldcg(reinterpret_cast<const float4*>(base + (size_t)(t * p.splits + s2) * kTileBytes) +
                                  (size_t)row * (BN / 4) + q);
          acc.x += x.x; acc.y += x.y; acc.z += x.z; acc.w += x.w;
        }
      }
    }
    if (row < p.M) {
      T* o = out + (int64_t)row * p.so + t * BN + q * 4;
      o[0] = from_f32<T>(acc.x);
      o[1] = from_f32<T>(acc.y);
      o[2] = from_f32<T>(acc.z);
      o[3] = from_f32<T>(acc.w);
    }
  }
  fence_before();
  __syncthreads();
  if (tid == 0) epochs[c] = e;
  if (warp == 0) {
    fence_after();
    tmem_dealloc(tmem, BN);
  }
}

}  // namespace
}  // namespace mvb

extern "C" size_t mvb_linear_allreduce_buffer_bytes(void) { return mvb::kDataOff + 2 * mvb::kSlotBytes; }

extern "C" int mvb_linear_allreduce(const mvb_allreduce_peers* peers, const mvb_tensor* x, const mvb_tensor* w,
                                    mvb_tensor* out, void* stream) {
  using namespace mvb;
  const char* op = "linear_allreduce";
  MVB_CHECK_ARG(peers != nullptr && x != nullptr && w != nullptr && out != nullptr, "%s: NULL argument", op);
  MVB_CHECK_ARG(peers->world >= 1 && peers->world <= kMaxRanks && peers->rank >= 0 && peers->rank < peers->world,
                "%s: world %d / rank %d out of range (1..%d ranks)", op, peers->world, peers->rank, kMaxRanks);
  MVB_CHECK_ARG(peers->buf_bytes >= kDataOff + 2 * kSlotBytes, "%s: buffers smaller than %zu bytes", op,
                (size_t)(kDataOff + 2 * kSlotBytes));
  for (int r = 0; r < peers->world; ++r)
    MVB_CHECK_ARG(peers->bufs[r] != nullptr && (reinterpret_cast<uintptr_t>(peers->bufs[r]) & 255) == 0,
                  "%s: buffer of rank %d is NULL or not 256-byte aligned", op, r);
  int rc;
  if ((rc = check_tensor(x, op, "x", 2)) || (rc = check_tensor(w, op, "w", 2)) || (rc = check_tensor(out, op, "out", 2)))
    return rc;
  const int64_t M = x->shape[0], K = x->shape[1], N = w->shape[0];
  MVB_CHECK_ARG(w->shape[1] == K && out->shape[0] == M && out->shape[1] == N, "%s: x [M, K], w [N, K], out [M, N]", op);
  MVB_CHECK_ARG(x->dtype == w->dtype && x->dtype == out->dtype, "%s: x, w and out must share one dtype", op);
  MVB_CHECK_SUPPORTED(x->dtype == MVB_BF16 || x->dtype == MVB_F16, "%s: bf16/fp16 only", op);
  MVB_CHECK_SUPPORTED(M <= BM, "%s: at most %d rows (decode batches)", op, BM);
  MVB_CHECK_SUPPORTED(N % BN == 0 && kCtas % (N / BN) == 0, "%s: N must be 64 x a divisor of %d", op, kCtas);
  const int tiles = (int)(N / BN), splits = kCtas / tiles;
  MVB_CHECK_SUPPORTED(K % (BK * splits) == 0, "%s: K = %lld must be a multiple of %d", op, (long long)K, BK * splits);
  MVB_CHECK_SUPPORTED(x->stride[1] == 1 && w->stride[1] == 1 && out->stride[1] == 1 && x->stride[0] % 8 == 0 &&
                          w->stride[0] % 8 == 0 && aligned16(x->data) && aligned16(w->data),
                      "%s: rows must be contiguous and 16-byte aligned", op);
  if (M == 0) return MVB_OK;
  LaParams p;
  memset(&p, 0, sizeof(p));
  const cuuint32_t box_x[2] = {(cuuint32_t)BK, (cuuint32_t)BM}, box_w[2] = {(cuuint32_t)BK, (cuuint32_t)BN};
  const cuuint64_t dx[2] = {(cuuint64_t)K, (cuuint64_t)M}, dw[2] = {(cuuint64_t)K, (cuuint64_t)N};
  const cuuint64_t sx[1] = {(cuuint64_t)x->stride[0] * 2}, sw[1] = {(cuuint64_t)w->stride[0] * 2};
  if (!tma::encode(&p.tm_x, x->dtype, 2, x->data, dx, sx, box_x) || !tma::encode(&p.tm_w, w->dtype, 2, w->data, dw, sw, box_w))
    MVB_FAIL(MVB_ERR_CUDA, "%s: the TMA descriptors could not be built", op);
  for (int r = 0; r < peers->world; ++r) p.bufs[r] = static_cast<char*>(peers->bufs[r]);
  p.out = out->data;
  p.so = out->stride[0];
  p.M = (int)M; p.N = (int)N; p.world = peers->world; p.rank = peers->rank;
  p.splits = splits;
  p.kb_per_split = (int)(K / BK / splits);
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (x->dtype == MVB_BF16) {
    static unsigned long long mask = 0;
    ensure_smem_attr(linear_allreduce_kernel<__nv_bfloat16>, SMEM, mask);
    linear_allreduce_kernel<__nv_bfloat16><<<kCtas, kThreads, SMEM, st>>>(p);
  } else {
    static unsigned long long mask = 0;
    ensure_smem_attr(linear_allreduce_kernel<__half>, SMEM, mask);
    linear_allreduce_kernel<__half><<<kCtas, kThreads, SMEM, st>>>(p);
  }
  MVB_CHECK_LAUNCH(op);
  return MVB_OK;
}
