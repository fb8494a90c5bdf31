// Chunked GDN prefill that allocates nothing: the two-launch prefill of
// wkvm_chunk_gated_delta_rule with its workspace in a fixed array that the
// library itself carries in device memory.
//
// Who needs it: hosts that reach this library through the bare C ABI and
// cannot allocate device memory on the call path -- for example a runtime
// whose device memory is all owned by its own pool allocator, or an embedding
// (cgo, JNI) with no allocator of its own, where a cudaMalloc would also
// synchronise the device in the middle of serving.
//
// The array is kGdnScratchBytes (64 MiB) on every GPU that loads the library,
// held until the process exits. Requests are processed in windows of chunks
// that fit it; one window must hold one chunk record plus the carried state
// for every (sequence, value head), so nseq * HV is limited to about 480.
#include <mutex>

#include "common.cuh"

namespace wkvm {

int gdn_two_phase(const void* q, const void* k, const void* v, const void* g, const void* beta,
                  void* o, const float* h_in, float* h_out, bool slots, const int32_t* ids,
                  int64_t num_slots, const int64_t* cu, int nseq, int T, int H, int HV,
                  float scale, bool l2norm, int dtype, void* workspace, int64_t ws_bytes,
                  int* status, cudaStream_t stream);

namespace {

constexpr int64_t kGdnScratchBytes = int64_t(64) << 20;
static __device__ __align__(256) uint8_t g_gdn_scratch[kGdnScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_ptr[kMaxDevices] = {};
unsigned long long g_scratch_ctx[kMaxDevices] = {};

// cuCtxGetId of the current context (0 if the driver cannot say), fetched
// through the runtime so the library needs no link against libcuda.
using CtxGetCurrentFn = int (*)(void**);
using CtxGetIdFn = int (*)(void*, unsigned long long*);

unsigned long long current_context_id() {
  static CtxGetCurrentFn get_current = nullptr;
  static CtxGetIdFn get_id = nullptr;
  static bool looked_up = false;
  if (!looked_up) {
    looked_up = true;
    cudaDriverEntryPointQueryResult q1, q2;
    void* f1 = nullptr;
    void* f2 = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f1, cudaEnableDefault, &q1) == cudaSuccess &&
        cudaGetDriverEntryPoint("cuCtxGetId", &f2, cudaEnableDefault, &q2) == cudaSuccess &&
        q1 == cudaDriverEntryPointSuccess && q2 == cudaDriverEntryPointSuccess) {
      get_current = reinterpret_cast<CtxGetCurrentFn>(f1);
      get_id = reinterpret_cast<CtxGetIdFn>(f2);
    }
  }
  void* ctx = nullptr;
  unsigned long long id = 0;
  if (get_current && get_id && get_current(&ctx) == 0 && ctx) get_id(ctx, &id);
  return id;
}

// Device address of g_gdn_scratch on the current device, looked up once per
// device and context (the host-side symbol is not a device address). A new
// context on the device (after cudaDeviceReset) is looked up afresh.
int scratch_address(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return WKVM_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return WKVM_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  const unsigned long long ctx = current_context_id();
  if (!g_scratch_ptr[dev] || g_scratch_ctx[dev] != ctx) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_gdn_scratch) != cudaSuccess || !p) return WKVM_ERR_CUDA;
    g_scratch_ptr[dev] = p;
    g_scratch_ctx[dev] = ctx;
  }
  *out = g_scratch_ptr[dev];
  return WKVM_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace
}  // namespace wkvm

extern "C" int64_t wkvm_gdn_chunk_workspace_bytes(int32_t, int32_t, int32_t, int32_t, int32_t);

extern "C" int wkvm_chunk_gated_delta_rule_static(
    const void* q, const void* k, const void* v, const void* g, const void* beta, void* o,
    const float* h0, float* ht, const int64_t* cu_seqlens, int32_t B, int32_t T, int32_t H,
    int32_t HV, int32_t K, int32_t V, float scale, int32_t use_qk_l2norm, int32_t dtype,
    int32_t* status, wkvm_stream_t stream) {
  if (K != 128 || V != 128) return WKVM_ERR_SHAPE;
  const int act = dtype & ~WKVM_GATES_F32;
  if (act != WKVM_DTYPE_BF16 && act != WKVM_DTYPE_F16) return WKVM_ERR_DTYPE;
  if (B < 0 || T < 0 || H <= 0 || HV <= 0 || HV % H) return WKVM_ERR_INVALID_ARG;
  if (B == 0) return WKVM_OK;
  if (!q || !k || !v || !g || !beta || !o) return WKVM_ERR_INVALID_ARG;
  if (!wkvm::aligned16(q) || !wkvm::aligned16(k) || !wkvm::aligned16(v) ||
      !wkvm::aligned16(o) || (h0 && !wkvm::aligned16(h0)) || (ht && !wkvm::aligned16(ht)))
    return WKVM_ERR_ALIGN;
  // whole prefill in one window, or at least one chunk per window plus the
  // state carried between windows
  const int64_t full = wkvm_gdn_chunk_workspace_bytes(B, T, HV, K, V);
  const int64_t one_window = (int64_t)B * HV * K * V * 4 + 256 +
                             wkvm_gdn_chunk_workspace_bytes(B, 1, HV, K, V);
  if (full > wkvm::kGdnScratchBytes && one_window > wkvm::kGdnScratchBytes)
    return WKVM_ERR_SCRATCH;
  void* ws = nullptr;
  const int rc = wkvm::scratch_address(&ws);
  if (rc != WKVM_OK) return rc;
  return wkvm::gdn_two_phase(q, k, v, g, beta, o, h0, ht, false, nullptr, 0, cu_seqlens, B, T, H,
                             HV, scale, use_qk_l2norm != 0, dtype, ws, wkvm::kGdnScratchBytes,
                             status, (cudaStream_t)stream);
}
