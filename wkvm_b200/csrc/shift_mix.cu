// Token shift + lerp ("addcmul") prologue of the RWKV-7 time-mix and
// channel-mix blocks for single-token decode, with the token-shift state read
// and written in place in the arena by slot id.
//
// For row b (slot s = ids[b]) and channel d:
//   delta = bf16(shift[s][d] - x[b][d])          (fla token_shift, decode)
//   out_i[b][d] = x[b][d] + delta * mix_i[d]      (torch.addcmul, i < n_mix)
//   shift[s][d] = x[b][d]                         (the new token-shift state)
// Replaces fla/modules/token_shift.py:521 (token_shift with a cache) followed by
// fla/ops/rwkv7/fused_addcmul.py:290 (torch_addcmul_rwkv7, the decode path)
// and the x.addcmul(delta, x_k) of RWKV7FeedForward
// (fla/models/rwkv7/modeling_rwkv7.py:98-115), plus wkvm's per-step
// gather/scatter of the shift family (wkvm/runner/state.py:63-97).
// Pure streaming: 16-byte loads and stores, one thread per 8 channels.
#include "common.cuh"

namespace wkvm {
namespace {

constexpr int kMaxMix = 6;

struct MixArgs {
  const void* x;
  void* out;        // [n_mix, B, D]
  uint8_t* shift;   // slot rows, slot_stride bytes apart
  int64_t slot_stride;
  int64_t num_slots;
  const int32_t* ids;
  const void* mix[kMaxMix];
  int n_mix, B, D;
  int* status;
};

template <typename T>
__global__ void __launch_bounds__(256) shift_mix_kernel(MixArgs p) {
  const int D8 = p.D >> 3;
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= (int64_t)p.B * D8) return;
  const int b = (int)(e / D8), d0 = (int)(e - (int64_t)b * D8) * 8;
  // every load that does not depend on the slot id goes out first
  const int32_t s = p.ids[b];
  const uint4 xu = *reinterpret_cast<const uint4*>(static_cast<const T*>(p.x) + (int64_t)b * p.D + d0);
  uint4 mu[kMaxMix];
#pragma unroll
  for (int m = 0; m < kMaxMix; ++m)
    if (m < p.n_mix) mu[m] = *reinterpret_cast<const uint4*>(static_cast<const T*>(p.mix[m]) + d0);
  if (s < 0 || (int64_t)s >= p.num_slots) {
    if (d0 == 0) report(p.status, WKVM_ERR_SLOT_RANGE);
    return;
  }
  uint4* srow = reinterpret_cast<uint4*>(p.shift + (int64_t)s * p.slot_stride + (int64_t)d0 * 2);
  const uint4 pu = *srow;
  const T* xe = reinterpret_cast<const T*>(&xu);
  const T* pe = reinterpret_cast<const T*>(&pu);
  float xv[8], dv[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    xv[i] = to_f32(xe[i]);
    dv[i] = to_f32(from_f32<T>(__fsub_rn(to_f32(pe[i]), xv[i])));  // delta is stored 16-bit
  }
  *srow = xu;
#pragma unroll
  for (int m = 0; m < kMaxMix; ++m) {
    if (m >= p.n_mix) break;
    const T* me = reinterpret_cast<const T*>(&mu[m]);
    uint4 ou;
    T* oe = reinterpret_cast<T*>(&ou);
#pragma unroll
    for (int i = 0; i < 8; ++i) oe[i] = from_f32<T>(__fadd_rn(xv[i], __fmul_rn(dv[i], to_f32(me[i]))));
    *reinterpret_cast<uint4*>(static_cast<T*>(p.out) + ((int64_t)m * p.B + b) * p.D + d0) = ou;
  }
}

bool al16(const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; }

}  // namespace
}  // namespace wkvm

extern "C" int wkvm_wkv7_shift_mix_slots(const void* x, void* out, void* shift_rows,
                                         int64_t slot_stride, int64_t num_slots,
                                         const int32_t* slot_ids, const void* const* mixes,
                                         int32_t n_mix, int32_t B, int32_t D, int32_t dtype,
                                         int32_t* status, wkvm_stream_t stream) {
  if (B < 0 || D <= 0 || n_mix < 0 || n_mix > wkvm::kMaxMix || num_slots <= 0)
    return WKVM_ERR_INVALID_ARG;
  if (B == 0) return WKVM_OK;
  if (!x || !shift_rows || !slot_ids || (n_mix > 0 && (!out || !mixes)))
    return WKVM_ERR_INVALID_ARG;
  if (dtype != WKVM_DTYPE_BF16 && dtype != WKVM_DTYPE_F16) return WKVM_ERR_DTYPE;
  if (D % 8) return WKVM_ERR_SHAPE;
  if (!wkvm::al16(x) || !wkvm::al16(shift_rows) || (n_mix > 0 && !wkvm::al16(out)) ||
      slot_stride % 16)
    return WKVM_ERR_ALIGN;
  wkvm::MixArgs a{x, out, static_cast<uint8_t*>(shift_rows), slot_stride, num_slots, slot_ids,
                  {}, n_mix, B, D, status};
  for (int m = 0; m < n_mix; ++m) {
    if (!mixes[m] || !wkvm::al16(mixes[m])) return WKVM_ERR_ALIGN;
    a.mix[m] = mixes[m];
  }
  const int64_t n = (int64_t)B * (D / 8);
  const int blocks = (int)((n + 255) / 256);
  if (dtype == WKVM_DTYPE_BF16)
    wkvm::shift_mix_kernel<__nv_bfloat16><<<blocks, 256, 0, (cudaStream_t)stream>>>(a);
  else
    wkvm::shift_mix_kernel<__half><<<blocks, 256, 0, (cudaStream_t)stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? WKVM_OK : WKVM_ERR_CUDA;
}
