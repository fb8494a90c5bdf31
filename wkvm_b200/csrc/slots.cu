// Slot row movement: fork (copy), zero, snapshot (gather to a packed buffer,
// possibly pinned host memory), restore (scatter from it) and live migration
// (peer stores into another GPU's bank).
//
// A state family tensor is viewed as [outer, num_slots, row]. One launch moves
// n slots x outer rows. Each CTA moves a 16 KiB stripe of one (pair, outer)
// row with 128-bit loads and stores; stripes are laid out so consecutive CTAs
// walk consecutive addresses of a row.
#include "common.cuh"

namespace wkvm {
namespace {

constexpr int kMoveThreads = 256;
constexpr int kVecPerThread = 4;                                      // 4 x 16 B
constexpr int64_t kStripeBytes = (int64_t)kMoveThreads * kVecPerThread * 16;  // 16 KiB

struct MoveArgs {
  const char* src;      // nullptr => write zeros
  char* dst;
  int64_t src_outer_stride, src_slot_stride;
  int64_t dst_outer_stride, dst_slot_stride;
  int64_t row_bytes;
  int64_t outer;
  const int32_t* src_ids;  // nullptr => identity (packed buffer index)
  const int32_t* dst_ids;
  int64_t src_limit, dst_limit;
  int64_t stripes_per_row;
  int* status;
};

__global__ void __launch_bounds__(kMoveThreads) slot_move_kernel(MoveArgs a) {
  const int64_t stripe = blockIdx.x % a.stripes_per_row;
  const int64_t oi = blockIdx.x / a.stripes_per_row;  // outer index
  const int64_t pair = blockIdx.y;
  if (oi >= a.outer) return;
  int64_t s_row = pair, d_row = pair;
  if (a.src_ids) s_row = a.src_ids[pair];
  if (a.dst_ids) d_row = a.dst_ids[pair];
  if ((a.src && (s_row < 0 || s_row >= a.src_limit)) || d_row < 0 || d_row >= a.dst_limit) {
    if (threadIdx.x == 0 && stripe == 0 && oi == 0) report(a.status, WKVM_ERR_SLOT_RANGE);
    return;
  }
  const int64_t off0 = stripe * kStripeBytes;
  char* d = a.dst + oi * a.dst_outer_stride + d_row * a.dst_slot_stride;
  const char* s = a.src ? a.src + oi * a.src_outer_stride + s_row * a.src_slot_stride : nullptr;
  uint4 buf[kVecPerThread];
#pragma unroll
  for (int i = 0; i < kVecPerThread; ++i) {
    const int64_t off = off0 + ((int64_t)i * kMoveThreads + threadIdx.x) * 16;
    if (off < a.row_bytes) {
      buf[i] = s ? *reinterpret_cast<const uint4*>(s + off) : make_uint4(0, 0, 0, 0);
    }
  }
#pragma unroll
  for (int i = 0; i < kVecPerThread; ++i) {
    const int64_t off = off0 + ((int64_t)i * kMoveThreads + threadIdx.x) * 16;
    if (off < a.row_bytes) *reinterpret_cast<uint4*>(d + off) = buf[i];
  }
}

bool al16(int64_t x) { return (x & 15) == 0; }
bool al16p(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int launch_move(MoveArgs a, int64_t n, cudaStream_t stream) {
  if (n < 0 || a.outer < 0 || a.row_bytes < 0) return WKVM_ERR_INVALID_ARG;
  if (n == 0 || a.outer == 0 || a.row_bytes == 0) return WKVM_OK;
  if (!a.dst) return WKVM_ERR_INVALID_ARG;
  if (!al16(a.row_bytes) || !al16(a.src_outer_stride) || !al16(a.src_slot_stride) ||
      !al16(a.dst_outer_stride) || !al16(a.dst_slot_stride) || !al16p(a.dst) ||
      (a.src && !al16p(a.src)))
    return WKVM_ERR_ALIGN;
  if (n > 65535) return WKVM_ERR_INVALID_ARG;
  a.stripes_per_row = (a.row_bytes + kStripeBytes - 1) / kStripeBytes;
  const int64_t gx = a.stripes_per_row * a.outer;
  if (gx > 0x7fffffffLL) return WKVM_ERR_INVALID_ARG;
  dim3 grid((unsigned)gx, (unsigned)n);
  slot_move_kernel<<<grid, kMoveThreads, 0, stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? WKVM_OK : WKVM_ERR_CUDA;
}

// out = fp32(c1 * a) + fp32(c2 * b) per element, rounded once more to the
// family's dtype; with b absent, out = fp32(c1 * a). Each product and the sum
// are rounded separately (no fused multiply-add) so the result is bitwise
// what torch computes for `((1 - w) * a.float() + w * b.float()).to(dtype)`
// and `(a.float() * alpha).to(dtype)`.
template <typename T>
__global__ void __launch_bounds__(256) slot_affine_kernel(char* base, int64_t outer,
                                                          int64_t outer_stride,
                                                          int64_t slot_stride, int64_t row_elems,
                                                          int64_t num_slots,
                                                          const int32_t* dst_ids,
                                                          const int32_t* a_ids,
                                                          const int32_t* b_ids, float c1,
                                                          float c2, int* status) {
  const int64_t pair = blockIdx.y;
  const int64_t d = dst_ids[pair], a = a_ids[pair], b = b_ids ? b_ids[pair] : 0;
  if (d < 0 || d >= num_slots || a < 0 || a >= num_slots || b < 0 || b >= num_slots) {
    if (threadIdx.x == 0 && blockIdx.x == 0) report(status, WKVM_ERR_SLOT_RANGE);
    return;
  }
  const int64_t total = outer * row_elems;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t o = e / row_elems, i = e - o * row_elems;
    char* ob = base + o * outer_stride;
    const float x = to_f32(reinterpret_cast<const T*>(ob + a * slot_stride)[i]);
    float y = __fmul_rn(c1, x);
    if (b_ids) y = __fadd_rn(y, __fmul_rn(c2, to_f32(reinterpret_cast<const T*>(ob + b * slot_stride)[i])));
    reinterpret_cast<T*>(ob + d * slot_stride)[i] = from_f32<T>(y);
  }
}

}  // namespace
}  // namespace wkvm

using wkvm::MoveArgs;

extern "C" int wkvm_slot_affine(void* base, int64_t outer, int64_t outer_stride,
                                int64_t slot_stride, int64_t row_bytes, int64_t num_slots,
                                const int32_t* dst_ids, const int32_t* a_ids,
                                const int32_t* b_ids, int32_t n, float c1, float c2,
                                int32_t dtype, int32_t* status, wkvm_stream_t stream) {
  if (!base || (n > 0 && (!dst_ids || !a_ids))) return WKVM_ERR_INVALID_ARG;
  if (n < 0 || outer < 0 || row_bytes < 0 || n > 65535) return WKVM_ERR_INVALID_ARG;
  if (n == 0 || outer == 0 || row_bytes == 0) return WKVM_OK;
  const int es = dtype == WKVM_DTYPE_F32 ? 4 : 2;
  if (row_bytes % es) return WKVM_ERR_ALIGN;
  const int64_t row_elems = row_bytes / es;
  const int64_t total = outer * row_elems;
  int64_t blocks = (total + 255) / 256;
  if (blocks > 1184) blocks = 1184;  // 8 resident blocks on each of 148 SMs
  dim3 grid((unsigned)blocks, (unsigned)n);
  cudaStream_t st = (cudaStream_t)stream;
  switch (dtype) {
    case WKVM_DTYPE_F32:
      wkvm::slot_affine_kernel<float><<<grid, 256, 0, st>>>((char*)base, outer, outer_stride,
          slot_stride, row_elems, num_slots, dst_ids, a_ids, b_ids, c1, c2, status);
      break;
    case WKVM_DTYPE_BF16:
      wkvm::slot_affine_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>((char*)base, outer,
          outer_stride, slot_stride, row_elems, num_slots, dst_ids, a_ids, b_ids, c1, c2, status);
      break;
    case WKVM_DTYPE_F16:
      wkvm::slot_affine_kernel<__half><<<grid, 256, 0, st>>>((char*)base, outer, outer_stride,
          slot_stride, row_elems, num_slots, dst_ids, a_ids, b_ids, c1, c2, status);
      break;
    default:
      return WKVM_ERR_DTYPE;
  }
  return cudaGetLastError() == cudaSuccess ? WKVM_OK : WKVM_ERR_CUDA;
}

extern "C" int wkvm_slot_copy(void* base, int64_t outer, int64_t outer_stride,
                              int64_t slot_stride, int64_t row_bytes, int64_t num_slots,
                              const int32_t* src_ids, const int32_t* dst_ids, int32_t n,
                              int32_t* status, wkvm_stream_t stream) {
  if (!base || (n > 0 && (!src_ids || !dst_ids))) return WKVM_ERR_INVALID_ARG;
  MoveArgs a{(const char*)base, (char*)base, outer_stride, slot_stride, outer_stride,
             slot_stride, row_bytes, outer, src_ids, dst_ids, num_slots, num_slots, 0, status};
  return wkvm::launch_move(a, n, (cudaStream_t)stream);
}

extern "C" int wkvm_slot_zero(void* base, int64_t outer, int64_t outer_stride,
                              int64_t slot_stride, int64_t row_bytes, int64_t num_slots,
                              const int32_t* ids, int32_t n, int32_t* status,
                              wkvm_stream_t stream) {
  if (!base || (n > 0 && !ids)) return WKVM_ERR_INVALID_ARG;
  MoveArgs a{nullptr, (char*)base, 0, 0, outer_stride, slot_stride, row_bytes, outer,
             nullptr, ids, 0, num_slots, 0, status};
  return wkvm::launch_move(a, n, (cudaStream_t)stream);
}

extern "C" int wkvm_slot_snapshot(const void* base, int64_t outer, int64_t outer_stride,
                                  int64_t slot_stride, int64_t row_bytes, int64_t num_slots,
                                  const int32_t* ids, int32_t n, void* packed,
                                  int32_t* status, wkvm_stream_t stream) {
  if (!base || !packed || (n > 0 && !ids)) return WKVM_ERR_INVALID_ARG;
  MoveArgs a{(const char*)base, (char*)packed, outer_stride, slot_stride, row_bytes,
             outer * row_bytes, row_bytes, outer, ids, nullptr, num_slots, (int64_t)n, 0,
             status};
  return wkvm::launch_move(a, n, (cudaStream_t)stream);
}

extern "C" int wkvm_slot_restore(void* base, int64_t outer, int64_t outer_stride,
                                 int64_t slot_stride, int64_t row_bytes, int64_t num_slots,
                                 const int32_t* ids, int32_t n, const void* packed,
                                 int32_t* status, wkvm_stream_t stream) {
  if (!base || !packed || (n > 0 && !ids)) return WKVM_ERR_INVALID_ARG;
  MoveArgs a{(const char*)packed, (char*)base, row_bytes, outer * row_bytes, outer_stride,
             slot_stride, row_bytes, outer, nullptr, ids, (int64_t)n, num_slots, 0, status};
  return wkvm::launch_move(a, n, (cudaStream_t)stream);
}

extern "C" int wkvm_slot_gather(const void* base, int64_t outer, int64_t outer_stride,
                                int64_t slot_stride, int64_t row_bytes, int64_t num_slots,
                                const int32_t* ids, int32_t n, void* dst,
                                int64_t dst_outer_stride, int64_t dst_index_stride,
                                int32_t* status, wkvm_stream_t stream) {
  if (!base || !dst || (n > 0 && !ids)) return WKVM_ERR_INVALID_ARG;
  MoveArgs a{(const char*)base, (char*)dst, outer_stride, slot_stride, dst_outer_stride,
             dst_index_stride, row_bytes, outer, ids, nullptr, num_slots, (int64_t)n, 0, status};
  return wkvm::launch_move(a, n, (cudaStream_t)stream);
}

extern "C" int wkvm_slot_scatter(void* base, int64_t outer, int64_t outer_stride,
                                 int64_t slot_stride, int64_t row_bytes, int64_t num_slots,
                                 const int32_t* ids, int32_t n, const void* src,
                                 int64_t src_outer_stride, int64_t src_index_stride,
                                 int32_t* status, wkvm_stream_t stream) {
  if (!base || !src || (n > 0 && !ids)) return WKVM_ERR_INVALID_ARG;
  MoveArgs a{(const char*)src, (char*)base, src_outer_stride, src_index_stride, outer_stride,
             slot_stride, row_bytes, outer, nullptr, ids, (int64_t)n, num_slots, 0, status};
  return wkvm::launch_move(a, n, (cudaStream_t)stream);
}

extern "C" int wkvm_slot_migrate(const void* src_base, void* dst_base, int64_t outer,
                                 int64_t outer_stride, int64_t slot_stride, int64_t row_bytes,
                                 int64_t src_num_slots, int64_t dst_num_slots,
                                 const int32_t* src_ids, const int32_t* dst_ids, int32_t n,
                                 int32_t* status, wkvm_stream_t stream) {
  if (!src_base || !dst_base || (n > 0 && (!src_ids || !dst_ids))) return WKVM_ERR_INVALID_ARG;
  MoveArgs a{(const char*)src_base, (char*)dst_base, outer_stride, slot_stride, outer_stride,
             slot_stride, row_bytes, outer, src_ids, dst_ids, src_num_slots, dst_num_slots, 0,
             status};
  return wkvm::launch_move(a, n, (cudaStream_t)stream);
}

extern "C" int wkvm_enable_peer_access(int32_t device, int32_t peer) {
  int prev = 0;
  WKVM_CUDA_TRY(cudaGetDevice(&prev));
  int can = 0;
  WKVM_CUDA_TRY(cudaDeviceCanAccessPeer(&can, device, peer));
  if (!can) return WKVM_ERR_UNSUPPORTED;
  WKVM_CUDA_TRY(cudaSetDevice(device));
  cudaError_t e = cudaDeviceEnablePeerAccess(peer, 0);
  if (e == cudaErrorPeerAccessAlreadyEnabled) {
    (void)cudaGetLastError();  // clear the sticky-free status of this benign error
    e = cudaSuccess;
  }
  cudaSetDevice(prev);
  return e == cudaSuccess ? WKVM_OK : WKVM_ERR_CUDA;
}

extern "C" int wkvm_version(void) { return 100; }

extern "C" const char* wkvm_strerror(int code) {
  switch (code) {
    case WKVM_OK: return "ok";
    case WKVM_ERR_INVALID_ARG: return "invalid argument";
    case WKVM_ERR_SHAPE: return "unsupported shape";
    case WKVM_ERR_DTYPE: return "unsupported dtype";
    case WKVM_ERR_SLOT_RANGE: return "slot id out of range";
    case WKVM_ERR_DUPLICATE: return "duplicate slot id in batch";
    case WKVM_ERR_CUDA: return "CUDA runtime error";
    case WKVM_ERR_ALIGN: return "pointer or size not 16-byte aligned";
    case WKVM_ERR_UNSUPPORTED: return "unsupported option";
    case WKVM_ERR_TIMEOUT: return "bounded wait timed out";
    case WKVM_ERR_SCRATCH: return "request larger than the static scratch array";
    default: return "unknown error";
  }
}
