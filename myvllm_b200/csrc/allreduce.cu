// One-shot all-reduce over NVLink peer memory, for the decode-size partial sums that the
// row-parallel output projections exchange (reference m/layers/linear.py:159-164, where
// RowParallelLinear calls dist.all_reduce).  Every rank owns one buffer, allocated by
// mvb_ipc_alloc and mapped into the other ranks' processes through CUDA IPC:
//
//   [0, 4096)      flags   uint32 [2 slots][8 source ranks][64 blocks], written by the peers
//   [4096, 4352)   epochs  uint32 [64 blocks], this rank's per-block call counters
//   [8192, ...)    data    2 slots x max_bytes
//
// Every launch runs all kBlocks (64) blocks, whatever the message size; block b owns bytes
// [b chunk, (b+1) chunk) of the message (chunk = ceil(bytes / 64), rounded to 16 B; a block
// whose range is empty still takes part) and synchronises only with block b of the other
// ranks:
//   1. copy this rank's chunk of the input into its own slot (e & 1), e = epoch + 1;
//   2. store e into flags[slot][rank][b] of every peer (release, system scope), after the
//      block's copy;
//   3. wait (acquire, bounded) until every peer's flags[slot][peer][b] on this rank read e;
//   4. read the chunk from every rank's slot, sum in fp32 in rank order (so every rank
//      gets the same bits) and write the output chunk.
// Because every block runs on every call, the per-block call counters stay equal and all
// blocks of a call use the same slot.  Two slots alternate: a rank starts call e+2 only
// after its call e+1 finished, in which it saw a flag of call e+1 from every peer; a peer
// stores those only after its own call e finished reading (kernels on one stream run in
// order), so no peer still reads the slot that call e+2 overwrites, whatever the sizes of
// the calls.  The counters live in device memory, so a captured CUDA graph replays
// correctly.  Nothing here uses multicast; peer data moves by plain loads.  A wait that
// gives up sets the device error word, and that block writes this rank's own input into
// its part of out (a defined value, not the sum) so the caller can detect it through
// mvb_device_status.
#include "common.cuh"
#include "tcgen05.cuh"  // report_device_error

namespace mvb {
namespace {

constexpr int kMaxRanks = MVB_AR_MAX_RANKS;
constexpr int kBlocks = 64;  // blocks of every launch (and flag slots per rank)
constexpr int kThreads = 512;
constexpr size_t kFlagsOff = 0, kEpochOff = 4096, kDataOff = 8192;
constexpr uint32_t kSpinLimit = 1u << 22;  // polls with a short sleep each: about two seconds
constexpr int kErrAllReduce = 5;

struct ArParams {
  char* bufs[kMaxRanks];
  const void* inp;
  void* out;
  size_t max_bytes, nbytes, chunk;
  int world, rank;
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

template <typename T>
__global__ void __launch_bounds__(kThreads) allreduce_oneshot_kernel(const __grid_constant__ ArParams p) {
  __shared__ uint32_t s_epoch;
  __shared__ int s_fail;
  const int b = blockIdx.x, tid = threadIdx.x;
  char* mine = p.bufs[p.rank];
  uint32_t* epochs = reinterpret_cast<uint32_t*>(mine + kEpochOff);
  if (tid == 0) {
    s_epoch = epochs[b] + 1;
    s_fail = 0;
  }
  __syncthreads();
  const uint32_t e = s_epoch;
  const int slot = e & 1;
  const size_t beg = (size_t)b * p.chunk < p.nbytes ? (size_t)b * p.chunk : p.nbytes;
  const size_t end = beg + p.chunk < p.nbytes ? beg + p.chunk : p.nbytes;
  const char* in = static_cast<const char*>(p.inp);
  const size_t slot_off = kDataOff + (size_t)slot * p.max_bytes;

  // 1. this rank's chunk into its own slot, for the peers to read
  for (size_t i = beg + (size_t)tid * 16; i < end; i += (size_t)kThreads * 16)
    *reinterpret_cast<uint4*>(mine + slot_off + i) = *reinterpret_cast<const uint4*>(in + i);
  __syncthreads();

  // 2. publish (the fence orders the whole block's copy, seen through the barrier, before the
  //    flag store) and 3. wait for every peer
  const int peer = tid;
  if (peer < p.world && peer != p.rank) {
    __threadfence_system();
    st_release_sys(reinterpret_cast<uint32_t*>(p.bufs[peer] + kFlagsOff) + (slot * kMaxRanks + p.rank) * kBlocks + b,
                   e);
    const uint32_t* f = reinterpret_cast<const uint32_t*>(mine + kFlagsOff) + (slot * kMaxRanks + peer) * kBlocks + b;
    uint32_t it = 0;
    while (ld_acquire_sys(f) != e) {
      if (++it == kSpinLimit) {
        s_fail = 1;
        report_device_error(kErrAllReduce);
        break;
      }
      __nanosleep(64);
    }
  }
  __syncthreads();

  // 4. the sum, in rank order (after a failed wait: this rank's own input)
  const bool failed = s_fail != 0;
  for (size_t i = beg + (size_t)tid * 16; i < end; i += (size_t)kThreads * 16) {
    const uint4 own = *reinterpret_cast<const uint4*>(in + i);
    if (failed) {
      *reinterpret_cast<uint4*>(static_cast<char*>(p.out) + i) = own;
      continue;
    }
    // every peer load is in flight before the first add: the NVLink round trips overlap
    uint4 u[kMaxRanks];
#pragma unroll
    for (int r = 0; r < kMaxRanks; ++r)
      if (r < p.world) u[r] = r == p.rank ? own : __ldcg(reinterpret_cast<const uint4*>(p.bufs[r] + slot_off + i));
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int r = 0; r < kMaxRanks; ++r) {
      if (r < p.world) {
        float f[8];
        unpack8<T>(u[r], f);
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] += f[j];
      }
    }
    *reinterpret_cast<uint4*>(static_cast<char*>(p.out) + i) = pack8<T>(acc);
  }
  if (tid == 0) epochs[b] = e;
}

}  // namespace
}  // namespace mvb

extern "C" size_t mvb_allreduce_buffer_bytes(size_t max_message_bytes) {
  const size_t m = (max_message_bytes + 255) / 256 * 256;
  return mvb::kDataOff + 2 * m;
}

extern "C" int mvb_ipc_alloc(size_t bytes, void** dev_ptr, void* handle) {
  MVB_CHECK_ARG(dev_ptr != nullptr && handle != nullptr && bytes > mvb::kDataOff, "ipc_alloc: bad arguments");
  void* ptr = nullptr;
  cudaError_t e = cudaMalloc(&ptr, bytes);
  if (e != cudaSuccess) MVB_FAIL(MVB_ERR_CUDA, "ipc_alloc: cudaMalloc(%zu): %s", bytes, cudaGetErrorString(e));
  e = cudaMemset(ptr, 0, bytes);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, ptr);
  if (e != cudaSuccess) {
    cudaFree(ptr);
    MVB_FAIL(MVB_ERR_CUDA, "ipc_alloc: %s", cudaGetErrorString(e));
  }
  memcpy(handle, &h, sizeof(h));
  *dev_ptr = ptr;
  return MVB_OK;
}

extern "C" int mvb_ipc_free(void* dev_ptr) {
  const cudaError_t e = cudaFree(dev_ptr);
  if (e != cudaSuccess) MVB_FAIL(MVB_ERR_CUDA, "ipc_free: %s", cudaGetErrorString(e));
  return MVB_OK;
}

extern "C" int mvb_ipc_open(const void* handle, void** dev_ptr) {
  MVB_CHECK_ARG(handle != nullptr && dev_ptr != nullptr, "ipc_open: bad arguments");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) MVB_FAIL(MVB_ERR_CUDA, "ipc_open: %s", cudaGetErrorString(e));
  return MVB_OK;
}

extern "C" int mvb_ipc_close(void* dev_ptr) {
  const cudaError_t e = cudaIpcCloseMemHandle(dev_ptr);
  if (e != cudaSuccess) MVB_FAIL(MVB_ERR_CUDA, "ipc_close: %s", cudaGetErrorString(e));
  return MVB_OK;
}

extern "C" int mvb_allreduce_oneshot(const mvb_allreduce_peers* peers, const mvb_tensor* inp, mvb_tensor* out,
                                     void* stream) {
  using namespace mvb;
  const char* op = "allreduce_oneshot";
  MVB_CHECK_ARG(peers != nullptr && inp != nullptr && out != nullptr, "%s: NULL argument", op);
  MVB_CHECK_ARG(peers->world >= 2 && peers->world <= kMaxRanks && peers->rank >= 0 && peers->rank < peers->world,
                "%s: world %d / rank %d out of range (2..%d ranks)", op, peers->world, peers->rank, kMaxRanks);
  for (int r = 0; r < peers->world; ++r)
    MVB_CHECK_ARG(peers->bufs[r] != nullptr && (reinterpret_cast<uintptr_t>(peers->bufs[r]) & 255) == 0,
                  "%s: buffer of rank %d is NULL or not 256-byte aligned", op, r);
  MVB_CHECK_ARG(peers->buf_bytes > kDataOff, "%s: buffer too small", op);
  MVB_CHECK_SUPPORTED(inp->dtype == MVB_BF16 || inp->dtype == MVB_F16, "%s: bf16/f16 only", op);
  MVB_CHECK_ARG(out->dtype == inp->dtype && numel(out) == numel(inp), "%s: out must match inp", op);
  const int64_t n = numel(inp);
  // contiguous tensors of any rank
  auto contiguous = [](const mvb_tensor* t) {
    int64_t expect = 1;
    for (int d = t->ndim - 1; d >= 0; --d) {
      if (t->shape[d] != 1 && t->stride[d] != expect) return false;
      expect *= t->shape[d];
    }
    return true;
  };
  MVB_CHECK_SUPPORTED(contiguous(inp) && contiguous(out), "%s: contiguous tensors only", op);
  const size_t nbytes = (size_t)n * 2;
  const size_t max_bytes = (peers->buf_bytes - kDataOff) / 2 / 256 * 256;
  MVB_CHECK_ARG(nbytes <= max_bytes, "%s: %zu bytes exceed the buffer's %zu-byte slots", op, nbytes, max_bytes);
  MVB_CHECK_SUPPORTED(nbytes % 16 == 0 && aligned16(inp->data) && aligned16(out->data),
                      "%s: sizes and pointers must be 16-byte multiples", op);
  if (nbytes == 0) return MVB_OK;
  ArParams p;
  memset(&p, 0, sizeof(p));
  for (int r = 0; r < peers->world; ++r) p.bufs[r] = static_cast<char*>(peers->bufs[r]);
  p.inp = inp->data;
  p.out = out->data;
  p.max_bytes = max_bytes;
  p.nbytes = nbytes;
  p.world = peers->world;
  p.rank = peers->rank;
  // always kBlocks blocks (see the header comment): the partition may change with the size,
  // the slot each call uses may not
  p.chunk = ((nbytes + kBlocks - 1) / kBlocks + 15) / 16 * 16;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (inp->dtype == MVB_BF16)
    allreduce_oneshot_kernel<__nv_bfloat16><<<kBlocks, kThreads, 0, st>>>(p);
  else
    allreduce_oneshot_kernel<__half><<<kBlocks, kThreads, 0, st>>>(p);
  MVB_CHECK_LAUNCH(op);
  return MVB_OK;
}
