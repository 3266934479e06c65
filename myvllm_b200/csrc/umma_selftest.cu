// Built-in self-test of the tensor-core layer (tcgen05.cuh): one CTA computes
//   D[128, N] = A B1 + (negate ? -1 : 1) A B2        (fp16 operands, fp32 accumulate)
// with A and B staged in either 128-byte-swizzle layout (K-major or MN-major), exactly
// as the GDN and attention kernels stage theirs.  Exported so that a deployment can
// check the descriptors on its GPU (tests/test_gpu_umma.py) before trusting the kernels.
#include "tcgen05.cuh"

namespace mvb {
namespace {

struct SelftestParams {
  const __half *a, *b1, *b2;
  float* d;
  int n, k, a_mn, b_mn, negate;
};

// Stage a [rows x K] (K-major, storage [rows][K]) or [K x rows] (MN-major, storage
// [K][rows]) fp16 operand into the swizzled shared layout.
__device__ void stage(char* dst, const __half* src, int rows, int K, bool mn) {
  if (!mn) {
    for (int i = threadIdx.x; i < rows * (K / 8); i += blockDim.x) {
      const int r = i / (K / 8), c = i % (K / 8);
      *reinterpret_cast<uint4*>(dst + (c >> 3) * rows * 128 + umma::sw128(r, c & 7)) =
          *reinterpret_cast<const uint4*>(src + (size_t)r * K + c * 8);
    }
  } else {
    for (int i = threadIdx.x; i < K * (rows / 8); i += blockDim.x) {
      const int kr = i / (rows / 8), c = i % (rows / 8);
      *reinterpret_cast<uint4*>(dst + (c >> 3) * K * 128 + umma::sw128(kr, c & 7)) =
          *reinterpret_cast<const uint4*>(src + (size_t)kr * rows + c * 8);
    }
  }
}

__global__ void __launch_bounds__(128, 1) umma_selftest_kernel(SelftestParams p) {
  extern __shared__ __align__(1024) char smem_raw[];
  char* smem = umma::align1024(smem_raw);
  __shared__ uint64_t mbar;
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;
  const int M = 128, N = p.n, K = p.k;
  char* sA = smem;
  char* sB1 = sA + M * K * 2;
  char* sB2 = sB1 + N * K * 2;
  const int warp = threadIdx.x >> 5;

  stage(sA, p.a, M, K, p.a_mn);
  stage(sB1, p.b1, N, K, p.b_mn);
  stage(sB2, p.b2, N, K, p.b_mn);
  if (threadIdx.x == 0) {
    umma::mbar_init(&mbar, 1);
    umma::mbar_fence_init();
    abort_flag = 0;
  }
  if (warp == 0) umma::tmem_alloc(&tmem_slot, 128);
  umma::fence_async_smem();
  umma::fence_before();
  __syncthreads();
  umma::fence_after();
  const uint32_t tbase = tmem_slot;

  if (threadIdx.x == 0) {
    const uint32_t id1 = umma::idesc_f16(M, N, p.a_mn, p.b_mn, false);
    const uint32_t id2 = umma::idesc_f16(M, N, p.a_mn, p.b_mn, p.negate != 0);
    const uint32_t a0 = smem_u32(sA), b10 = smem_u32(sB1), b20 = smem_u32(sB2);
    for (int pass = 0; pass < 2; ++pass) {
      for (int ks = 0; ks < K / 16; ++ks) {
        const uint64_t da = p.a_mn ? umma::desc_mnmajor(a0, K * 128, ks) : umma::desc_kmajor(a0, M, ks);
        const uint32_t bb = pass == 0 ? b10 : b20;
        const uint64_t db = p.b_mn ? umma::desc_mnmajor(bb, K * 128, ks) : umma::desc_kmajor(bb, N, ks);
        umma::mma_f16(tbase, da, db, pass == 0 ? id1 : id2, pass > 0 || ks > 0);
      }
    }
    umma::commit(&mbar);
  }
  if (!umma::mbar_wait(&mbar, 0)) {
    abort_flag = 1;
    report_device_error(1);
  }
  umma::fence_after();
  __syncthreads();
  if (!abort_flag) {
    const int row = threadIdx.x;  // warp w reads TMEM lanes 32w..32w+31
    for (int c = 0; c < N; c += 16) {
      float v[16];
      umma::tmem_ld16(umma::taddr(tbase, warp * 32, c), v);
      umma::tmem_wait_ld();
      for (int j = 0; j < 16; ++j) p.d[(size_t)row * N + c + j] = v[j];
    }
  }
  umma::fence_before();
  __syncthreads();
  if (warp == 0) umma::tmem_dealloc(tbase, 128);
}

}  // namespace
}  // namespace mvb

extern "C" int mvb_selftest_umma(const void* a, const void* b1, const void* b2, float* d, int n, int k, int a_mn,
                                 int b_mn, int negate, void* stream) {
  using namespace mvb;
  MVB_CHECK_ARG(a && b1 && b2 && d, "selftest_umma: null pointer");
  MVB_CHECK_ARG((n == 64 || n == 128) && (k == 64 || k == 128), "selftest_umma: N, K must be 64 or 128");
  SelftestParams p{static_cast<const __half*>(a), static_cast<const __half*>(b1), static_cast<const __half*>(b2), d,
                   n, k, a_mn, b_mn, negate};
  const int smem = (128 * k + 2 * n * k) * 2 + 1024;
  cudaFuncSetAttribute(umma_selftest_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  umma_selftest_kernel<<<1, 128, smem, static_cast<cudaStream_t>(stream)>>>(p);
  MVB_CHECK_LAUNCH("selftest_umma");
  return MVB_OK;
}

