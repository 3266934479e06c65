// Minimal sm_100a tensor-core layer: TMEM allocation, UMMA shared-memory and instruction
// descriptors, tcgen05.mma issue/commit, TMEM loads/stores and bounded mbarrier waits.
//
// Operand tiles live in shared memory in the 128-byte-swizzle canonical layouts:
//   K-major  (rows = M or N, K contiguous): per 64-element K half a [rows][128 B] block;
//            16-byte chunk c of row r sits at r*128 + ((c ^ (r & 7)) << 4); blocks are
//            1024-byte aligned; SBO = 1024 B (8-row group stride), LBO unused (1).
//   MN-major (rows = K, MN contiguous): per 64-element MN block a [K][128 B] block with the
//            same swizzle; SBO = 1024 B (8 K-rows), LBO = byte stride between MN blocks.
// The same XOR swizzle is what cp.async stores produce when they address chunks with
// sw128(); so tiles staged by plain copies are directly UMMA operands.
#pragma once

#include "common.cuh"

namespace mvb {
namespace umma {

// ------------------------------------------------------------------ layouts ----
__device__ __forceinline__ uint32_t sw128(int r, int c) { return r * 128 + ((c ^ (r & 7)) << 4); }

// Byte offset of element (row, col) of a 16-bit tile stored as 64-column blocks of
// [rows][128 B] (block stride `block_bytes`).
__device__ __forceinline__ uint32_t elem_off(int row, int col, uint32_t block_bytes) {
  return (col >> 6) * block_bytes + sw128(row, (col >> 3) & 7) + ((col & 7) << 1);
}

// The 128-byte swizzle is a function of absolute shared-memory address bits, so operand
// tiles must start on 1024-byte boundaries: kernels over-allocate dynamic shared memory
// by 1 KB and round the base up with this.
__device__ __forceinline__ char* align1024(char* p) {
  const uint32_t a = smem_u32(p);
  return p + (((a + 1023u) & ~1023u) - a);
}

// ------------------------------------------------------------- descriptors ----
// Shared-memory matrix descriptor, SWIZZLE_128B, version 1 (sm100).
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;  // version
  d |= (uint64_t)2 << 61;  // SWIZZLE_128B
  return d;
}

// K-major operand with `rows` rows; k-step ks covers K elements [16 ks, 16 ks + 16).
__device__ __forceinline__ uint64_t desc_kmajor(uint32_t base, int rows, int ks) {
  const uint32_t a = base + (ks >> 2) * (uint32_t)(rows * 128) + (ks & 3) * 32;
  return smem_desc(a, 16, 1024);
}
// MN-major operand stored as [K rows][64-col blocks], block stride `block_bytes`;
// k-step ks covers K rows [16 ks, 16 ks + 16).
__device__ __forceinline__ uint64_t desc_mnmajor(uint32_t base, uint32_t block_bytes, int ks) {
  return smem_desc(base + ks * 2048, block_bytes, 1024);
}

// Instruction descriptor, kind::f16: fp16 (or bf16) A/B, fp32 accumulator.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N, bool a_mn, bool b_mn, bool a_neg = false,
                                                 bool bf16 = false) {
  return (1u << 4)                                   // D = f32
         | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10)  // A, B format
         | ((a_neg ? 1u : 0u) << 13) | ((a_mn ? 1u : 0u) << 15) | ((b_mn ? 1u : 0u) << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// ------------------------------------------------------------------ issue ----
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                        bool accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate ? 1 : 0));
}

// A operand in tensor memory: lane m holds row m of A, K-major, two 16-bit elements per
// 32-bit column (the even K index in the low half); k-step ks of a K = 16 MMA starts at
// column a_tmem + 8 ks.  The instruction descriptor must say K-major for A.
__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                           bool accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate ? 1 : 0));
}

// Arrive on `mbar` once every MMA this thread issued so far has completed.
__device__ __forceinline__ void commit(uint64_t* mbar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(mbar))
               : "memory");
}

__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// generic-proxy shared-memory writes -> visible to the tensor core (async proxy)
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// ------------------------------------------------------------------- TMEM ----
// Warp-collective.  Writes the allocated base address to *slot.
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
               "r"(ncols));
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}

// 32 lanes x 32 bits, 16 consecutive columns per thread.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t* r = reinterpret_cast<uint32_t*>(v);
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float* v) {
  const uint32_t* r = reinterpret_cast<const uint32_t*>(v);
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// TMEM address of (lane, column).
__device__ __forceinline__ uint32_t taddr(uint32_t base, int lane, int col) {
  return base + ((uint32_t)lane << 16) + (uint32_t)col;
}

// --------------------------------------------------------------- mbarrier ----
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

// Waits for the phase with parity `phase` to complete.  Gives up after `max_iter` polls
// (each poll may suspend the thread for a hardware-defined time) and returns false.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t phase, uint32_t max_iter = (1u << 22)) {
  const uint32_t a = smem_u32(bar);
  for (uint32_t i = 0; i < max_iter; ++i) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(done)
        : "r"(a), "r"(phase)
        : "memory");
    if (done) return true;
  }
  return false;
}

}  // namespace umma

// Per translation unit: set (never cleared by kernels) when a bounded wait inside a kernel
// gave up.  Every unit registers a host reader, and mvb_device_status() reads and clears
// all of them.
namespace {
__device__ int g_mvb_device_error = 0;

__device__ __forceinline__ void report_device_error(int code) { atomicMax(&g_mvb_device_error, code); }

int read_device_error(int* out) {
  int zero = 0;
  cudaError_t e = cudaMemcpyFromSymbol(out, g_mvb_device_error, sizeof(int));
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_mvb_device_error, &zero, sizeof(int));
  return e == cudaSuccess ? 0 : -1;
}

struct DeviceErrorReader {
  DeviceErrorReader() { register_status_reader(&read_device_error); }
};
const DeviceErrorReader g_device_error_reader;
}  // namespace

}  // namespace mvb
