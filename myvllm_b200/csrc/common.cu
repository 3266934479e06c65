// Status plumbing shared by every entry point of libmyvllm_b200.
#include <vector>

#include "common.cuh"

namespace mvb {

static thread_local char g_last_error[512] = "";

constexpr int kPathOps = 3;  // MVB_OP_CHUNK_GDN, MVB_OP_FA_PREFILL, MVB_OP_PAGED_PREFILL
static thread_local int g_path[kPathOps] = {MVB_PATH_NONE, MVB_PATH_NONE, MVB_PATH_NONE};
static thread_local char g_path_reason[kPathOps][160] = {"", "", ""};

void set_path(int op, int path, const char* reason) {
  if (op < 0 || op >= kPathOps) return;
  g_path[op] = path;
  snprintf(g_path_reason[op], sizeof(g_path_reason[op]), "%s", reason ? reason : "");
}

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

int check_tensor(const mvb_tensor* t, const char* op, const char* name, int ndim) {
  if (t == nullptr) MVB_FAIL(MVB_ERR_ARG, "%s: %s is NULL", op, name);
  // ndim < 0: any rank from 1 to 6 (the caller checks the rank it needs)
  if (ndim < 0 ? (t->ndim < 1 || t->ndim > 6) : t->ndim != ndim)
    MVB_FAIL(MVB_ERR_ARG, "%s: %s must have %d dims, got %d", op, name, ndim, t->ndim);
  ndim = t->ndim;
  for (int i = 0; i < ndim; ++i)
    if (t->shape[i] < 0) MVB_FAIL(MVB_ERR_ARG, "%s: %s has a negative extent", op, name);
  if (numel(t) > 0 && t->data == nullptr) MVB_FAIL(MVB_ERR_ARG, "%s: %s has no data pointer", op, name);
  return MVB_OK;
}

static std::vector<StatusReader>& status_readers() {
  static std::vector<StatusReader> v;
  return v;
}

void register_status_reader(StatusReader f) { status_readers().push_back(f); }

int read_all_status(int* out) {
  int worst = 0;
  for (StatusReader f : status_readers()) {
    int s = 0;
    if (f(&s) != 0) return -1;
    worst = s > worst ? s : worst;
  }
  *out = worst;
  return 0;
}

int num_sms() {
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n;
}

}  // namespace mvb

extern "C" {

int mvb_version(void) { return 100; }

const char* mvb_last_error(void) { return mvb::g_last_error; }

int mvb_last_path(int op, const char** reason) {
  if (op < 0 || op >= mvb::kPathOps) {
    if (reason) *reason = "unknown op";
    return -1;
  }
  if (reason) *reason = mvb::g_path_reason[op];
  return mvb::g_path[op];
}

int mvb_device_status(int* status) {
  if (status == nullptr) MVB_FAIL(MVB_ERR_ARG, "device_status: null pointer");
  if (mvb::read_all_status(status) != 0) MVB_FAIL(MVB_ERR_CUDA, "device_status: reading the error words failed");
  return MVB_OK;
}

}  // extern "C"
