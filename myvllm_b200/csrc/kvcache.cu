// Paged KV-cache write: k/v [T, Hkv, D] -> caches [n_blocks, block_size, Hkv, D] at
// slot_mapping[t] (slot = block * block_size + offset, -1 = skip).
//
// The reference has no such kernel (the slot_mapping field is only sketched in
// m/utils/context.py:15); the cache layout is the one its paged attention reads
// (m/ops/full_attention.py:186-195).  A pure copy: each warp moves one (token, head)
// row with 16-byte accesses; rows are streamed with evict-first stores.
#include "common.cuh"

namespace mvb {
namespace {

struct KvParams {
  const char *k, *v;
  char *kc, *vc;
  const int32_t* slots;
  int64_t sk_t, sk_h, sv_t, sv_h;              // bytes
  int64_t skc_b, skc_t, skc_h, svc_b, svc_t, svc_h;  // bytes
  int T, hkv, block_size, krow_bytes, vrow_bytes, n_blocks;
};

// One warp per (token, head); rows are copied in 16-byte units.
__global__ void __launch_bounds__(256) store_kv_kernel(KvParams p) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= p.T * p.hkv) return;
  const int t = warp / p.hkv, h = warp % p.hkv;
  const int slot = p.slots[t];
  if (slot < 0) return;
  const int64_t b = slot / p.block_size, o = slot % p.block_size;
  if (b >= p.n_blocks) return;  // out-of-range slot: the host validates where it can
  const uint4* ks = reinterpret_cast<const uint4*>(p.k + t * p.sk_t + h * p.sk_h);
  uint4* kd = reinterpret_cast<uint4*>(p.kc + b * p.skc_b + o * p.skc_t + h * p.skc_h);
  for (int i = lane; i < p.krow_bytes / 16; i += 32) __stcs(kd + i, __ldcs(ks + i));
  const uint4* vs = reinterpret_cast<const uint4*>(p.v + t * p.sv_t + h * p.sv_h);
  uint4* vd = reinterpret_cast<uint4*>(p.vc + b * p.svc_b + o * p.svc_t + h * p.svc_h);
  for (int i = lane; i < p.vrow_bytes / 16; i += 32) __stcs(vd + i, __ldcs(vs + i));
}

}  // namespace
}  // namespace mvb

extern "C" int mvb_store_kvcache(const mvb_tensor* k, const mvb_tensor* v, mvb_tensor* k_cache,
                                 mvb_tensor* v_cache, const mvb_tensor* slot_mapping, void* stream) {
  using namespace mvb;
  const char* op = "store_kvcache";
  int rc;
  if ((rc = check_tensor(k, op, "k", 3)) || (rc = check_tensor(v, op, "v", 3)) ||
      (rc = check_tensor(k_cache, op, "k_cache", 4)) || (rc = check_tensor(v_cache, op, "v_cache", 4)) ||
      (rc = check_tensor(slot_mapping, op, "slot_mapping", 1)))
    return rc;
  const int64_t T = k->shape[0], hkv = k->shape[1], d = k->shape[2], dv = v->shape[2];
  MVB_CHECK_ARG(v->shape[0] == T && v->shape[1] == hkv, "%s: v must be [T, Hkv, Dv]", op);
  MVB_CHECK_ARG(slot_mapping->shape[0] == T && slot_mapping->dtype == MVB_I32, "%s: slot_mapping must be int32 [T]",
                op);
  MVB_CHECK_ARG(k_cache->shape[2] == hkv && k_cache->shape[3] == d && v_cache->shape[2] == hkv &&
                    v_cache->shape[3] == dv && k_cache->shape[1] == v_cache->shape[1] &&
                    k_cache->shape[0] == v_cache->shape[0],
                "%s: caches must be [n_blocks, block_size, Hkv, D]", op);
  MVB_CHECK_ARG(k->dtype == k_cache->dtype && v->dtype == v_cache->dtype && k->dtype == v->dtype,
                "%s: k/v and caches must share a dtype", op);
  const int es = dtype_size(k->dtype);
  MVB_CHECK_SUPPORTED(k->stride[2] == 1 && v->stride[2] == 1 && k_cache->stride[3] == 1 && v_cache->stride[3] == 1 &&
                          (d * es) % 16 == 0 && (dv * es) % 16 == 0 && aligned16(k->data) && aligned16(v->data) &&
                          aligned16(k_cache->data) && aligned16(v_cache->data) && (k->stride[0] * es) % 16 == 0 &&
                          (k->stride[1] * es) % 16 == 0 && (v->stride[0] * es) % 16 == 0 &&
                          (v->stride[1] * es) % 16 == 0 && (k_cache->stride[0] * es) % 16 == 0 &&
                          (k_cache->stride[1] * es) % 16 == 0 && (k_cache->stride[2] * es) % 16 == 0 &&
                          (v_cache->stride[0] * es) % 16 == 0 && (v_cache->stride[1] * es) % 16 == 0 &&
                          (v_cache->stride[2] * es) % 16 == 0,
                      "%s: rows must be contiguous and 16-byte aligned", op);
  if (T == 0 || hkv == 0) return MVB_OK;
  KvParams p;
  p.k = static_cast<const char*>(k->data); p.v = static_cast<const char*>(v->data);
  p.kc = static_cast<char*>(k_cache->data); p.vc = static_cast<char*>(v_cache->data);
  p.slots = static_cast<const int32_t*>(slot_mapping->data);
  p.sk_t = k->stride[0] * es; p.sk_h = k->stride[1] * es; p.sv_t = v->stride[0] * es; p.sv_h = v->stride[1] * es;
  p.skc_b = k_cache->stride[0] * es; p.skc_t = k_cache->stride[1] * es; p.skc_h = k_cache->stride[2] * es;
  p.svc_b = v_cache->stride[0] * es; p.svc_t = v_cache->stride[1] * es; p.svc_h = v_cache->stride[2] * es;
  p.T = (int)T; p.hkv = (int)hkv; p.block_size = (int)k_cache->shape[1];
  p.krow_bytes = (int)(d * es); p.vrow_bytes = (int)(dv * es); p.n_blocks = (int)k_cache->shape[0];
  const int64_t warps = T * hkv;
  const int threads = 256;
  const int64_t blocks = (warps * 32 + threads - 1) / threads;
  store_kv_kernel<<<(unsigned)blocks, threads, 0, static_cast<cudaStream_t>(stream)>>>(p);
  MVB_CHECK_LAUNCH(op);
  return MVB_OK;
}
