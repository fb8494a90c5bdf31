// Fused RWKV-7 time-mix decode core: everything fla's RWKV7Attention does
// between its projections and o_proj for one token, around the WKV update of
// an arena slot (fla/layers/rwkv7.py:270-349):
//
//   w  = -0.6065306597126334 * sigmoid(w_lora)       a = sigmoid(a_lora)
//   v  = lerp(v, v_first, sigmoid(v_lora))            (layers > 0)
//   kk = l2norm(k * k_k) per head (eps 1e-6)          k' = k + k (a - 1) k_a
//   h  = exp(w) h + (kk a) ((-kk)^T h) + k' v^T       o = h^T r      (in place)
//   o  = GroupNorm_head(o) * gn_w + gn_b               (eps = gn_eps)
//   o  = (o + (sum_head r k' r_k) v) * g
//
// One CTA per (slot, head) of 64 threads, state in registers exactly as the
// plain decode kernel (recurrent.cu); the gates and norms ride on the input
// staging and on the output, so a decode layer's ten small elementwise
// kernels of fla become part of the one that streams the state. Arithmetic
// is fp32 throughout (fla rounds each intermediate to the activation dtype).
#include "common.cuh"

namespace wkvm {
namespace {

constexpr int N = 64, ROWS = 16, CG = N / 4, RG = N / ROWS, NT = CG * RG;  // 64 threads
constexpr int kPreRows = 1;  // state rows a thread loads before an overlapped launch's wait

__device__ __forceinline__ float sigmoidf_(float x) { return 1.0f / (1.0f + __expf(-x)); }

__device__ __forceinline__ float wsum(float x) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) x += __shfl_xor_sync(0xffffffffu, x, off);
  return x;
}
// sum over the 16 lanes of a half-warp
__device__ __forceinline__ float hsum16(float x) {
#pragma unroll
  for (int off = 8; off > 0; off >>= 1) x += __shfl_xor_sync(0xffffffffu, x, off);
  return x;
}

struct TmArgs {
  const void *r, *w_raw, *k, *v, *v_first, *v_raw, *a_raw, *g;
  const void *k_k, *k_a, *r_k, *gn_w, *gn_b;
  void* o;
  float* bank;
  const int32_t* ids;
  int64_t num_slots;
  int H;
  float gn_eps;
  int* status;
  bool overlap;  // launched with programmatic dependent launch
};

template <typename T>
__global__ void __launch_bounds__(NT) wkv7_timemix_decode_kernel(TmArgs p) {
  __shared__ __align__(16) float s_in[6][N];  // 0 e^w, 1 -kk, 2 kk*a, 3 k', 4 r e^w, 5 v
  __shared__ __align__(16) float s_red[RG][2][N];
  __shared__ float s_dot[2][4];               // per staging warp: r.b, r.k', r.k'.r_k, |k k_k|^2
  __shared__ __align__(16) float s_ep[3][N];  // epilogue inputs: g, gn_w, gn_b

  const int H = p.H;
  const int n = blockIdx.x / H, hh = blockIdx.x - (blockIdx.x / H) * H;
  const int tid = threadIdx.x, cg = tid % CG, rg = tid / CG, lane = tid & 31, warp = tid >> 5;
  const int32_t id = p.ids[n];
  if (id < 0 || (int64_t)id >= p.num_slots) {
    if (tid == 0) report(p.status, WKVM_ERR_SLOT_RANGE);
    return;
  }
  const int64_t hoff = ((int64_t)id * H + hh) * (N * N);
  float4 hreg[ROWS];
  auto load_state = [&](int j0, int j1) {
    const float* src = p.bank + hoff + cg * 4;
#pragma unroll
    for (int j = 0; j < ROWS; ++j)
      if (j >= j0 && j < j1) hreg[j] = ld_stream_f4(src + (j * RG + rg) * N);
  };
  if (p.overlap) {
    // Overlapped launch: the CTA starts while the previous kernel in the
    // stream drains, sends out its first state row (which that kernel does
    // not write, by the opt-in's contract) and waits; the activations that
    // kernel may have produced are read after the wait, ahead of the other
    // state rows. More state before the wait delays the activations (the
    // gates are the first dependent chain) by more than it gains. The next
    // launch is released only after the wait, so no launch ever runs beside
    // a kernel older than its immediate predecessor.
    load_state(0, kPreRows);
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  }

  // ---- staging: thread e = tid owns channel e of this head
  const int64_t base = ((int64_t)n * H + hh) * N + tid;
  const int ch = hh * N + tid;  // channel within the layer
  const T* rp = static_cast<const T*>(p.r);
  const float rr = to_f32(rp[base]);
  const float wv = -0.6065306597126334f * sigmoidf_(to_f32(static_cast<const T*>(p.w_raw)[base]));
  const float kraw = to_f32(static_cast<const T*>(p.k)[base]);
  float vv = to_f32(static_cast<const T*>(p.v)[base]);
  if (p.v_first) {
    const float vf = to_f32(static_cast<const T*>(p.v_first)[base]);
    const float s = sigmoidf_(to_f32(static_cast<const T*>(p.v_raw)[base]));
    vv = fmaf(s, vf - vv, vv);
  }
  const float aa = sigmoidf_(to_f32(static_cast<const T*>(p.a_raw)[base]));
  const float kkr = kraw * to_f32(static_cast<const T*>(p.k_k)[ch]);
  const float kup = fmaf(kraw * (aa - 1.0f), to_f32(static_cast<const T*>(p.k_a)[ch]), kraw);
  const float rkk = to_f32(static_cast<const T*>(p.r_k)[ch]);
  // the epilogue's inputs are loaded now, with the rest of the staging
  s_ep[0][tid] = to_f32(static_cast<const T*>(p.g)[base]);
  s_ep[1][tid] = to_f32(static_cast<const T*>(p.gn_w)[ch]);
  s_ep[2][tid] = to_f32(static_cast<const T*>(p.gn_b)[ch]);
  // the (remaining) state rows go out after the activation loads they would
  // otherwise delay (the gates below are the first dependent chain)
  load_state(p.overlap ? kPreRows : 0, ROWS);
  // per-head sums: |k k_k|^2 first (kk needs it)
  float part_nn = wsum(kkr * kkr);
  if (lane == 0) s_dot[warp][3] = part_nn;
  __syncthreads();
  const float inv = 1.0f / sqrtf(s_dot[0][3] + s_dot[1][3] + 1e-6f);
  const float kk = kkr * inv;
  const float ew = __expf(wv);
  const float bb = kk * aa;
  s_in[0][tid] = ew;
  s_in[1][tid] = -kk;
  s_in[2][tid] = bb;
  s_in[3][tid] = kup;
  s_in[4][tid] = rr * ew;
  s_in[5][tid] = vv;
  {
    const float rb = wsum(rr * bb), rk = wsum(rr * kup), rkc = wsum(rr * kup * rkk);
    if (lane == 0) {
      s_dot[warp][0] = rb;
      s_dot[warp][1] = rk;
      s_dot[warp][2] = rkc;
    }
  }
  __syncthreads();

  // ---- WKV update (pre-update reductions, as the plain decode kernel)
  float4 pa = make_float4(0.f, 0.f, 0.f, 0.f), pr = pa;
#pragma unroll
  for (int j = 0; j < ROWS; ++j) {
    const int kr = j * RG + rg;
    const float a1 = s_in[1][kr], c4 = s_in[4][kr];
    pa.x = fmaf(a1, hreg[j].x, pa.x); pa.y = fmaf(a1, hreg[j].y, pa.y);
    pa.z = fmaf(a1, hreg[j].z, pa.z); pa.w = fmaf(a1, hreg[j].w, pa.w);
    pr.x = fmaf(c4, hreg[j].x, pr.x); pr.y = fmaf(c4, hreg[j].y, pr.y);
    pr.z = fmaf(c4, hreg[j].z, pr.z); pr.w = fmaf(c4, hreg[j].w, pr.w);
  }
  *reinterpret_cast<float4*>(&s_red[rg][0][cg * 4]) = pa;
  *reinterpret_cast<float4*>(&s_red[rg][1][cg * 4]) = pr;
  __syncthreads();
  float4 sa = make_float4(0.f, 0.f, 0.f, 0.f), ro = sa;
#pragma unroll
  for (int gi = 0; gi < RG; ++gi) {
    const float4 x = *reinterpret_cast<const float4*>(&s_red[gi][0][cg * 4]);
    const float4 y = *reinterpret_cast<const float4*>(&s_red[gi][1][cg * 4]);
    sa.x += x.x; sa.y += x.y; sa.z += x.z; sa.w += x.w;
    ro.x += y.x; ro.y += y.y; ro.z += y.z; ro.w += y.w;
  }
  const float rb = s_dot[0][0] + s_dot[1][0];
  const float rk = s_dot[0][1] + s_dot[1][1];
  const float corr = s_dot[0][2] + s_dot[1][2];
  const float4 v4 = *reinterpret_cast<const float4*>(&s_in[5][cg * 4]);
#pragma unroll
  for (int j = 0; j < ROWS; ++j) {
    const int kr = j * RG + rg;
    const float e = s_in[0][kr], bk = s_in[2][kr], ku = s_in[3][kr];
    hreg[j].x = fmaf(e, hreg[j].x, fmaf(bk, sa.x, ku * v4.x));
    hreg[j].y = fmaf(e, hreg[j].y, fmaf(bk, sa.y, ku * v4.y));
    hreg[j].z = fmaf(e, hreg[j].z, fmaf(bk, sa.z, ku * v4.z));
    hreg[j].w = fmaf(e, hreg[j].w, fmaf(bk, sa.w, ku * v4.w));
  }
  {
    float* dst = p.bank + hoff + cg * 4;
#pragma unroll
    for (int j = 0; j < ROWS; ++j) st_stream_f4(dst + (j * RG + rg) * N, hreg[j]);
  }

  // ---- epilogue on the 16 threads holding the head's 64 outputs (warp 0,
  //      lanes 0..15): GroupNorm over the head, correction, gate
  if (warp == 0) {
    float o4[4] = {fmaf(rk, v4.x, fmaf(rb, sa.x, ro.x)), fmaf(rk, v4.y, fmaf(rb, sa.y, ro.y)),
                   fmaf(rk, v4.z, fmaf(rb, sa.z, ro.z)), fmaf(rk, v4.w, fmaf(rb, sa.w, ro.w))};
    const float mean = hsum16(o4[0] + o4[1] + o4[2] + o4[3]) * (1.0f / N);
    float dv = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) dv = fmaf(o4[i] - mean, o4[i] - mean, dv);
    const float var = hsum16(dv) * (1.0f / N);
    const float rstd = 1.0f / sqrtf(var + p.gn_eps);
    if (rg == 0) {
      const float vals[4] = {v4.x, v4.y, v4.z, v4.w};
      T* op = static_cast<T*>(p.o) + ((int64_t)n * H + hh) * N + cg * 4;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int c = cg * 4 + i;
        const float gg = s_ep[0][c], gw = s_ep[1][c], gb = s_ep[2][c];
        const float on = fmaf((o4[i] - mean) * rstd, gw, gb);
        op[i] = from_f32<T>(fmaf(corr, vals[i], on) * gg);
      }
    }
  }
}

}  // namespace
}  // namespace wkvm

extern "C" int wkvm_wkv7_timemix_decode_slots(
    const void* r, const void* w_raw, const void* k, const void* v, const void* v_first,
    const void* v_raw, const void* a_raw, const void* g, const void* k_k, const void* k_a,
    const void* r_k, const void* gn_w, const void* gn_b, void* o, float* bank_layer,
    int64_t num_slots, const int32_t* slot_ids, int32_t B, int32_t H, int32_t K, float gn_eps,
    int32_t dtype, int32_t* status, wkvm_stream_t stream) {
  if (B < 0 || H <= 0) return WKVM_ERR_INVALID_ARG;
  if (B == 0) return WKVM_OK;
  if (!r || !w_raw || !k || !v || !a_raw || !g || !k_k || !k_a || !r_k || !gn_w || !gn_b || !o ||
      !bank_layer || !slot_ids || num_slots <= 0)
    return WKVM_ERR_INVALID_ARG;
  if ((v_first == nullptr) != (v_raw == nullptr)) return WKVM_ERR_INVALID_ARG;
  if (K != wkvm::N) return WKVM_ERR_SHAPE;
  if (reinterpret_cast<uintptr_t>(bank_layer) & 15u) return WKVM_ERR_ALIGN;
  const bool overlap = wkvm::decode_overlap();
  wkvm::TmArgs a{r, w_raw, k, v, v_first, v_raw, a_raw, g, k_k, k_a, r_k, gn_w, gn_b,
                 o, bank_layer, slot_ids, num_slots, H, gn_eps, status, overlap};
  void (*kern)(wkvm::TmArgs);
  switch (dtype) {
    case WKVM_DTYPE_BF16: kern = wkvm::wkv7_timemix_decode_kernel<__nv_bfloat16>; break;
    case WKVM_DTYPE_F16: kern = wkvm::wkv7_timemix_decode_kernel<__half>; break;
    case WKVM_DTYPE_F32: kern = wkvm::wkv7_timemix_decode_kernel<float>; break;
    default: return WKVM_ERR_DTYPE;
  }
  const dim3 grid((unsigned)((int64_t)B * H));
  cudaStream_t st = (cudaStream_t)stream;
  if (overlap) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(wkvm::NT);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, a) == cudaSuccess ? WKVM_OK : WKVM_ERR_CUDA;
  }
  kern<<<grid, wkvm::NT, 0, st>>>(a);
  return cudaGetLastError() == cudaSuccess ? WKVM_OK : WKVM_ERR_CUDA;
}
