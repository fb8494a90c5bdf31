// Recurrent (token-by-token) forms of the RWKV-7 DPLR rule and the gated
// delta rule, over fp32 state held in registers.
//
// One CTA owns one (sequence, head) state h[K][V]. Thread (rg, cg) holds the
// 4 columns [4cg, 4cg+4) of rows {j*RG + rg : j < ROWS} as float4 registers,
// so a warp's j-th load covers whole adjacent 256..512-byte rows (coalesced
// 128-bit loads) and the state is read from HBM once and written once per
// launch, whatever T is.
//
// Every column reduction the step needs is taken over the *pre-update* state
// in one pass, using the algebra of the update:
//   RWKV-7: h' = D h + b sa^T + k v^T, sa = a^T h, D = diag(exp w)
//           o  = h'^T r = (h^T (r*exp w)) + (r.b) sa + (r.k) v
//   GDN:    h' = e^g h + k v'^T, v' = beta (v - e^g h^T k)
//           o  = h'^T q = e^g (h^T q) + (q.k) v'
// so one barrier separates "read + partial sums" from "update + store".
#include "common.cuh"

namespace wkvm {

namespace {

constexpr int kMaxWarps = 8;

template <int NT>
__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) x += __shfl_xor_sync(0xffffffffu, x, off);
  return x;
}

__device__ __forceinline__ float4 f4_zero() { return make_float4(0.f, 0.f, 0.f, 0.f); }
__device__ __forceinline__ float4 f4_add(float4 a, float4 b) {
  return make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
}
__device__ __forceinline__ float4 f4_fma(float s, float4 x, float4 acc) {
  return make_float4(fmaf(s, x.x, acc.x), fmaf(s, x.y, acc.y), fmaf(s, x.z, acc.z),
                     fmaf(s, x.w, acc.w));
}

template <typename T>
__device__ __forceinline__ void store4(T* p, float4 x) {
  p[0] = from_f32<T>(x.x);
  p[1] = from_f32<T>(x.y);
  p[2] = from_f32<T>(x.z);
  p[3] = from_f32<T>(x.w);
}

// Resolves the state row of sequence n: slot id when `ids` is given, else n.
// Returns false (and reports) for an out-of-range id.
__device__ __forceinline__ bool state_row(const int32_t* ids, int64_t num_slots, int n,
                                          int64_t* row, int* status) {
  if (ids == nullptr) {
    *row = n;
    return true;
  }
  const int32_t id = ids[n];
  if (id < 0 || (int64_t)id >= num_slots) {
    if (threadIdx.x == 0) report(status, WKVM_ERR_SLOT_RANGE);
    return false;
  }
  *row = id;
  return true;
}

struct SeqRange {
  int64_t bos;
  int64_t len;
};

__device__ __forceinline__ SeqRange seq_range(const int64_t* cu_seqlens, int n, int T) {
  if (cu_seqlens) return {cu_seqlens[n], cu_seqlens[n + 1] - cu_seqlens[n]};
  return {(int64_t)n * T, (int64_t)T};
}

// ---------------------------------------------------------------------------
// RWKV-7 / DPLR. MUL_FORM: inputs (kk, a_gate) with a = -kk, b = kk * a_gate
// (fla fused_mul_recurrent_rwkv7, fused_recurrent.py:94-96); otherwise
// explicit (a, b) (fla fused_recurrent_dplr_delta_rule).
// ---------------------------------------------------------------------------
template <int N, int ROWS, typename Tin, bool MUL_FORM>
__global__ void __launch_bounds__((N / 4) * (N / ROWS))
wkv7_recurrent_kernel(const Tin* __restrict__ r, const Tin* __restrict__ w,
                      const Tin* __restrict__ k, const Tin* __restrict__ v,
                      const Tin* __restrict__ x5, const Tin* __restrict__ x6,
                      Tin* __restrict__ o, const float* h_in, float* h_out,
                      const int32_t* __restrict__ ids, int64_t num_slots,
                      const int64_t* __restrict__ cu_seqlens, int T, int H, float scale,
                      int* status) {
  constexpr int CG = N / 4;    // float4 column groups
  constexpr int RG = N / ROWS; // row groups
  constexpr int NT = CG * RG;
  constexpr int NW_IN = (N + 31) / 32;  // warps that stage one token's inputs
  static_assert(NT % 32 == 0 && NT / 32 <= kMaxWarps, "thread layout");

  // Per-token staged inputs (double-buffered by token parity):
  // 0 exp(w), 1 a, 2 b, 3 k, 4 r*scale*exp(w), 5 v
  __shared__ __align__(16) float s_in[2][6][N];
  __shared__ __align__(16) float s_red[2][RG][2][N];
  __shared__ float s_dot[2][NW_IN][2];

  const int nh = blockIdx.x;
  const int n = nh / H;
  const int hh = nh - n * H;
  const int tid = threadIdx.x;
  const int cg = tid % CG;
  const int rg = tid / CG;

  int64_t row = 0;
  if (!state_row(ids, num_slots, n, &row, status)) return;
  const int64_t hoff = (row * H + hh) * (int64_t)(N * N);
  const SeqRange sr = seq_range(cu_seqlens, n, T);

  float4 hreg[ROWS];
  if (h_in != nullptr) {
    const float* src = h_in + hoff + cg * 4;
#pragma unroll
    for (int j = 0; j < ROWS; ++j) hreg[j] = ld_stream_f4(src + (j * RG + rg) * N);
  } else {
#pragma unroll
    for (int j = 0; j < ROWS; ++j) hreg[j] = f4_zero();
  }

  // Token inputs are prefetched one step ahead into registers so the global
  // load latency of token t+1 overlaps the math of token t.
  Tin nx[6];
  auto fetch = [&](int64_t t) {
    const int64_t b = ((sr.bos + t) * H + hh) * (int64_t)N + tid;
    nx[0] = r[b];
    nx[1] = w[b];
    nx[2] = k[b];
    nx[3] = v[b];
    nx[4] = x5[b];
    nx[5] = x6[b];
  };
  // Programmatic dependent launch (opt-in for decode, see
  // wkvm_set_decode_overlap): the slot ids and the state were read above,
  // while the previous launch in the stream may still run; wait for it here,
  // before any input is read. Only after the wait does this CTA let the next
  // launch start, so at most two launches overlap: a launch can run beside
  // its immediate predecessor only, never beside an older one. Without the
  // launch attribute both instructions are no-ops.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (tid < N && sr.len > 0) fetch(0);

  for (int64_t t = 0; t < sr.len; ++t) {
    const int buf = (int)(t & 1);
    const int64_t base = ((sr.bos + t) * H + hh) * (int64_t)N;
    if (tid < N) {
      const float rr = to_f32(nx[0]) * scale;
      const float ew = expf(to_f32(nx[1]));
      const float kv = to_f32(nx[2]);
      const float vv = to_f32(nx[3]);
      const float p5 = to_f32(nx[4]);
      const float p6 = to_f32(nx[5]);
      if (t + 1 < sr.len) fetch(t + 1);
      const float aa = MUL_FORM ? -p5 : p5;
      const float bb = MUL_FORM ? p5 * p6 : p6;
      s_in[buf][0][tid] = ew;
      s_in[buf][1][tid] = aa;
      s_in[buf][2][tid] = bb;
      s_in[buf][3][tid] = kv;
      s_in[buf][4][tid] = rr * ew;
      s_in[buf][5][tid] = vv;
      float rb = warp_sum<32>(rr * bb);
      float rk = warp_sum<32>(rr * kv);
      if ((tid & 31) == 0) {
        s_dot[buf][tid >> 5][0] = rb;
        s_dot[buf][tid >> 5][1] = rk;
      }
    }
    __syncthreads();

    float4 pa = f4_zero(), pr = f4_zero();
#pragma unroll
    for (int j = 0; j < ROWS; ++j) {
      const int kr = j * RG + rg;
      pa = f4_fma(s_in[buf][1][kr], hreg[j], pa);
      pr = f4_fma(s_in[buf][4][kr], hreg[j], pr);
    }
    *reinterpret_cast<float4*>(&s_red[buf][rg][0][cg * 4]) = pa;
    *reinterpret_cast<float4*>(&s_red[buf][rg][1][cg * 4]) = pr;
    __syncthreads();

    float4 sa = f4_zero(), ro = f4_zero();
#pragma unroll
    for (int g = 0; g < RG; ++g) {
      sa = f4_add(sa, *reinterpret_cast<const float4*>(&s_red[buf][g][0][cg * 4]));
      ro = f4_add(ro, *reinterpret_cast<const float4*>(&s_red[buf][g][1][cg * 4]));
    }
    float rb = 0.f, rk = 0.f;
#pragma unroll
    for (int wi = 0; wi < NW_IN; ++wi) {
      rb += s_dot[buf][wi][0];
      rk += s_dot[buf][wi][1];
    }
    const float4 v4 = *reinterpret_cast<const float4*>(&s_in[buf][5][cg * 4]);

#pragma unroll
    for (int j = 0; j < ROWS; ++j) {
      const int kr = j * RG + rg;
      const float ew = s_in[buf][0][kr];
      const float bk = s_in[buf][2][kr];
      const float kk = s_in[buf][3][kr];
      float4 hn;
      hn.x = fmaf(ew, hreg[j].x, fmaf(bk, sa.x, kk * v4.x));
      hn.y = fmaf(ew, hreg[j].y, fmaf(bk, sa.y, kk * v4.y));
      hn.z = fmaf(ew, hreg[j].z, fmaf(bk, sa.z, kk * v4.z));
      hn.w = fmaf(ew, hreg[j].w, fmaf(bk, sa.w, kk * v4.w));
      hreg[j] = hn;
    }
    if (rg == 0) {
      float4 ov;
      ov.x = fmaf(rk, v4.x, fmaf(rb, sa.x, ro.x));
      ov.y = fmaf(rk, v4.y, fmaf(rb, sa.y, ro.y));
      ov.z = fmaf(rk, v4.z, fmaf(rb, sa.z, ro.z));
      ov.w = fmaf(rk, v4.w, fmaf(rb, sa.w, ro.w));
      store4(o + base + cg * 4, ov);
    }
  }

  if (h_out != nullptr) {
    float* dst = h_out + hoff + cg * 4;
#pragma unroll
    for (int j = 0; j < ROWS; ++j) st_stream_f4(dst + (j * RG + rg) * N, hreg[j]);
  }
}

// ---------------------------------------------------------------------------
// Gated delta rule (fla fused_recurrent_gated_delta_rule_fwd_kernel,
// fused_recurrent.py:28-170, head-wise g and beta, [K, V] state layout).
// ---------------------------------------------------------------------------
template <int K, int V, int ROWS, typename Tin>
__global__ void __launch_bounds__((V / 4) * (K / ROWS))
gdn_recurrent_kernel(const Tin* __restrict__ q, const Tin* __restrict__ k,
                     const Tin* __restrict__ v, const void* __restrict__ g,
                     const void* __restrict__ beta, Tin* __restrict__ o,
                     const float* h_in, float* h_out, const int32_t* __restrict__ ids,
                     int64_t num_slots, const int64_t* __restrict__ cu_seqlens, int T, int H,
                     int HV, float scale, bool l2norm, bool gates_f32, int* status) {
  constexpr int CG = V / 4;
  constexpr int RG = K / ROWS;
  constexpr int NT = CG * RG;
  constexpr int NW_IN = (K + 31) / 32;
  static_assert(NT % 32 == 0 && NT / 32 <= kMaxWarps, "thread layout");
  static_assert(NT >= K && NT >= V, "staging needs one thread per element");

  // 0 q, 1 k (raw), plus v
  __shared__ __align__(16) float s_qk[2][2][K];
  __shared__ __align__(16) float s_v[2][V];
  __shared__ __align__(16) float s_red[2][RG][2][V];
  __shared__ float s_dot[2][NW_IN][3];

  const int nh = blockIdx.x;
  const int n = nh / HV;
  const int hv = nh - n * HV;
  const int hq = hv / (HV / H);
  const int tid = threadIdx.x;
  const int cg = tid % CG;
  const int rg = tid / CG;

  int64_t row = 0;
  if (!state_row(ids, num_slots, n, &row, status)) return;
  const int64_t hoff = (row * HV + hv) * (int64_t)(K * V);
  const SeqRange sr = seq_range(cu_seqlens, n, T);

  float4 hreg[ROWS];
  if (h_in != nullptr) {
    const float* src = h_in + hoff + cg * 4;
#pragma unroll
    for (int j = 0; j < ROWS; ++j) hreg[j] = ld_stream_f4(src + (j * RG + rg) * V);
  } else {
#pragma unroll
    for (int j = 0; j < ROWS; ++j) hreg[j] = f4_zero();
  }

  // Inputs of token t+1 are fetched into registers while token t computes.
  Tin nq = Tin(), nk = Tin(), nv = Tin();
  float ng = 0.f, nb = 0.f;
  auto fetch = [&](int64_t t) {
    const int64_t tk = sr.bos + t;
    if (tid < K) {
      nq = q[(tk * H + hq) * (int64_t)K + tid];
      nk = k[(tk * H + hq) * (int64_t)K + tid];
    }
    if (tid < V) nv = v[(tk * HV + hv) * (int64_t)V + tid];
    ng = load_gate<Tin>(g, tk * HV + hv, gates_f32);
    nb = load_gate<Tin>(beta, tk * HV + hv, gates_f32);
  };
  if (sr.len > 0) fetch(0);

  for (int64_t t = 0; t < sr.len; ++t) {
    const int buf = (int)(t & 1);
    const int64_t tok = sr.bos + t;
    const int64_t v_base = (tok * HV + hv) * (int64_t)V;
    const float cur_v = to_f32(nv);
    const float cur_g = ng;
    const float cur_b = nb;
    const float qq = to_f32(nq);
    const float kv = to_f32(nk);
    if (t + 1 < sr.len) fetch(t + 1);
    if (tid < K) {
      s_qk[buf][0][tid] = qq;
      s_qk[buf][1][tid] = kv;
      const float d_qq = warp_sum<32>(qq * qq);
      const float d_kk = warp_sum<32>(kv * kv);
      const float d_qk = warp_sum<32>(qq * kv);
      if ((tid & 31) == 0) {
        s_dot[buf][tid >> 5][0] = d_qq;
        s_dot[buf][tid >> 5][1] = d_kk;
        s_dot[buf][tid >> 5][2] = d_qk;
      }
    }
    if (tid < V) s_v[buf][tid] = cur_v;
    const float eg = expf(cur_g);
    const float bt = cur_b;
    __syncthreads();

    float4 pk = f4_zero(), pq = f4_zero();
#pragma unroll
    for (int j = 0; j < ROWS; ++j) {
      const int kr = j * RG + rg;
      pq = f4_fma(s_qk[buf][0][kr], hreg[j], pq);
      pk = f4_fma(s_qk[buf][1][kr], hreg[j], pk);
    }
    *reinterpret_cast<float4*>(&s_red[buf][rg][0][cg * 4]) = pk;
    *reinterpret_cast<float4*>(&s_red[buf][rg][1][cg * 4]) = pq;
    __syncthreads();

    float4 hk = f4_zero(), hqv = f4_zero();
#pragma unroll
    for (int gi = 0; gi < RG; ++gi) {
      hk = f4_add(hk, *reinterpret_cast<const float4*>(&s_red[buf][gi][0][cg * 4]));
      hqv = f4_add(hqv, *reinterpret_cast<const float4*>(&s_red[buf][gi][1][cg * 4]));
    }
    float dqq = 0.f, dkk = 0.f, dqk = 0.f;
#pragma unroll
    for (int wi = 0; wi < NW_IN; ++wi) {
      dqq += s_dot[buf][wi][0];
      dkk += s_dot[buf][wi][1];
      dqk += s_dot[buf][wi][2];
    }
    const float inv_q = l2norm ? 1.0f / sqrtf(dqq + 1e-6f) : 1.0f;
    const float inv_k = l2norm ? 1.0f / sqrtf(dkk + 1e-6f) : 1.0f;
    const float qs = inv_q * scale;
    const float qk = dqk * qs * inv_k;  // (q*scale) . k after normalisation
    const float4 v4 = *reinterpret_cast<const float4*>(&s_v[buf][cg * 4]);
    const float egk = eg * inv_k;
    const float egq = eg * qs;
    float4 vn;  // v' = beta (v - e^g h^T k)
    vn.x = bt * fmaf(-egk, hk.x, v4.x);
    vn.y = bt * fmaf(-egk, hk.y, v4.y);
    vn.z = bt * fmaf(-egk, hk.z, v4.z);
    vn.w = bt * fmaf(-egk, hk.w, v4.w);

#pragma unroll
    for (int j = 0; j < ROWS; ++j) {
      const int kr = j * RG + rg;
      const float kn = s_qk[buf][1][kr] * inv_k;
      float4 hn;
      hn.x = fmaf(eg, hreg[j].x, kn * vn.x);
      hn.y = fmaf(eg, hreg[j].y, kn * vn.y);
      hn.z = fmaf(eg, hreg[j].z, kn * vn.z);
      hn.w = fmaf(eg, hreg[j].w, kn * vn.w);
      hreg[j] = hn;
    }
    if (rg == 0) {
      float4 ov;
      ov.x = fmaf(egq, hqv.x, qk * vn.x);
      ov.y = fmaf(egq, hqv.y, qk * vn.y);
      ov.z = fmaf(egq, hqv.z, qk * vn.z);
      ov.w = fmaf(egq, hqv.w, qk * vn.w);
      store4(o + v_base + cg * 4, ov);
    }
  }

  if (h_out != nullptr) {
    float* dst = h_out + hoff + cg * 4;
#pragma unroll
    for (int j = 0; j < ROWS; ++j) st_stream_f4(dst + (j * RG + rg) * V, hreg[j]);
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

struct RecArgs {
  const void *p0, *p1, *p2, *p3, *p4, *p5;
  void* o;
  const float* h_in;
  float* h_out;
  const int32_t* ids;
  int64_t num_slots;
  const int64_t* cu;
  int B, T, H, HV, K, V;
  float scale;
  bool l2norm;
  int* status;
  cudaStream_t stream;
  bool overlap = false;    // programmatic dependent launch (decode only)
  bool gates_f32 = false;  // GDN: g and beta are fp32 (WKVM_GATES_F32)
};

// Process-wide opt-in for overlapping consecutive decode launches.
bool g_decode_overlap = false;

template <int N, int ROWS, typename Tin, bool MUL>
int launch_wkv7_t(const RecArgs& a) {
  constexpr int NT = (N / 4) * (N / ROWS);
  dim3 grid((unsigned)((int64_t)a.B * a.H));
  if (a.overlap) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(NT);
    cfg.stream = a.stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(
        &cfg, wkv7_recurrent_kernel<N, ROWS, Tin, MUL>, (const Tin*)a.p0, (const Tin*)a.p1,
        (const Tin*)a.p2, (const Tin*)a.p3, (const Tin*)a.p4, (const Tin*)a.p5, (Tin*)a.o,
        a.h_in, a.h_out, a.ids, a.num_slots, a.cu, a.T, a.H, a.scale, a.status);
    return e == cudaSuccess ? WKVM_OK : WKVM_ERR_CUDA;
  }
  wkv7_recurrent_kernel<N, ROWS, Tin, MUL><<<grid, NT, 0, a.stream>>>(
      (const Tin*)a.p0, (const Tin*)a.p1, (const Tin*)a.p2, (const Tin*)a.p3,
      (const Tin*)a.p4, (const Tin*)a.p5, (Tin*)a.o, a.h_in, a.h_out, a.ids, a.num_slots,
      a.cu, a.T, a.H, a.scale, a.status);
  return cudaGetLastError() == cudaSuccess ? WKVM_OK : WKVM_ERR_CUDA;
}

template <typename Tin, bool MUL>
int launch_wkv7_n(const RecArgs& a) {
  switch (a.K) {
    case 32: return launch_wkv7_t<32, 8, Tin, MUL>(a);
    case 64: return launch_wkv7_t<64, 16, Tin, MUL>(a);
    case 128: return launch_wkv7_t<128, 16, Tin, MUL>(a);
    default: return WKVM_ERR_SHAPE;
  }
}

template <bool MUL>
int launch_wkv7(const RecArgs& a, int dtype) {
  switch (dtype) {
    case WKVM_DTYPE_F32: return launch_wkv7_n<float, MUL>(a);
    case WKVM_DTYPE_BF16: return launch_wkv7_n<__nv_bfloat16, MUL>(a);
    case WKVM_DTYPE_F16: return launch_wkv7_n<__half, MUL>(a);
    default: return WKVM_ERR_DTYPE;
  }
}

template <int K, int V, int ROWS, typename Tin>
int launch_gdn_t(const RecArgs& a) {
  constexpr int NT = (V / 4) * (K / ROWS);
  dim3 grid((unsigned)((int64_t)a.B * a.HV));
  gdn_recurrent_kernel<K, V, ROWS, Tin><<<grid, NT, 0, a.stream>>>(
      (const Tin*)a.p0, (const Tin*)a.p1, (const Tin*)a.p2, a.p3, a.p4, (Tin*)a.o, a.h_in,
      a.h_out, a.ids, a.num_slots, a.cu, a.T, a.H, a.HV, a.scale, a.l2norm, a.gates_f32,
      a.status);
  return cudaGetLastError() == cudaSuccess ? WKVM_OK : WKVM_ERR_CUDA;
}

template <typename Tin>
int launch_gdn_kv(const RecArgs& a) {
  if (a.K == 64 && a.V == 64) return launch_gdn_t<64, 64, 8, Tin>(a);
  if (a.K == 128 && a.V == 128) return launch_gdn_t<128, 128, 16, Tin>(a);
  return WKVM_ERR_SHAPE;
}

int launch_gdn(RecArgs a, int dtype) {
  a.gates_f32 = (dtype & WKVM_GATES_F32) != 0;
  switch (dtype & ~WKVM_GATES_F32) {
    case WKVM_DTYPE_F32: return launch_gdn_kv<float>(a);
    case WKVM_DTYPE_BF16: return launch_gdn_kv<__nv_bfloat16>(a);
    case WKVM_DTYPE_F16: return launch_gdn_kv<__half>(a);
    default: return WKVM_ERR_DTYPE;
  }
}

// Host-side checks shared by every recurrent entry point.
int check_common(const RecArgs& a, bool has_cu) {
  if (a.B < 0 || a.T < 0 || a.H <= 0 || a.K <= 0 || a.V <= 0) return WKVM_ERR_INVALID_ARG;
  if (!a.p0 || !a.p1 || !a.p2 || !a.p3 || !a.p4 || !a.p5 || !a.o) {
    if (a.B > 0 && a.T > 0) return WKVM_ERR_INVALID_ARG;
  }
  if ((a.h_in && !aligned16(a.h_in)) || (a.h_out && !aligned16(a.h_out))) return WKVM_ERR_ALIGN;
  (void)has_cu;
  return WKVM_OK;
}

}  // namespace

bool decode_overlap() { return g_decode_overlap; }

}  // namespace wkvm

using wkvm::RecArgs;

extern "C" int wkvm_fused_mul_recurrent_rwkv7(const void* r, const void* w, const void* k,
                                              const void* v, const void* kk, const void* a,
                                              void* o, const float* h0, float* ht,
                                              const int64_t* cu_seqlens, int32_t B, int32_t T,
                                              int32_t H, int32_t K, int32_t V, float scale,
                                              int32_t dtype, int32_t* status,
                                              wkvm_stream_t stream) {
  RecArgs args{r, w, k, v, kk, a, o, h0, ht, nullptr, 0, cu_seqlens, B, T, H, H, K, V,
               scale, false, status, (cudaStream_t)stream};
  int rc = wkvm::check_common(args, cu_seqlens != nullptr);
  if (rc) return rc;
  if (K != V) return WKVM_ERR_SHAPE;
  if (B == 0 || (T == 0 && cu_seqlens == nullptr)) {
    if (h0 && ht && h0 != ht) {
      WKVM_CUDA_TRY(cudaMemcpyAsync(ht, h0, (size_t)B * H * K * V * sizeof(float),
                                    cudaMemcpyDeviceToDevice, (cudaStream_t)stream));
    }
    return WKVM_OK;
  }
  return wkvm::launch_wkv7<true>(args, dtype);
}

extern "C" int wkvm_fused_recurrent_dplr(const void* r, const void* w, const void* k,
                                         const void* v, const void* a, const void* b, void* o,
                                         const float* h0, float* ht, const int64_t* cu_seqlens,
                                         int32_t B, int32_t T, int32_t H, int32_t K, int32_t V,
                                         float scale, int32_t dtype, int32_t* status,
                                         wkvm_stream_t stream) {
  RecArgs args{r, w, k, v, a, b, o, h0, ht, nullptr, 0, cu_seqlens, B, T, H, H, K, V,
               scale, false, status, (cudaStream_t)stream};
  int rc = wkvm::check_common(args, cu_seqlens != nullptr);
  if (rc) return rc;
  if (K != V) return WKVM_ERR_SHAPE;
  if (B == 0 || (T == 0 && cu_seqlens == nullptr)) {
    if (h0 && ht && h0 != ht) {
      WKVM_CUDA_TRY(cudaMemcpyAsync(ht, h0, (size_t)B * H * K * V * sizeof(float),
                                    cudaMemcpyDeviceToDevice, (cudaStream_t)stream));
    }
    return WKVM_OK;
  }
  return wkvm::launch_wkv7<false>(args, dtype);
}

extern "C" int wkvm_wkv7_decode_slots(const void* r, const void* w, const void* k,
                                      const void* v, const void* kk, const void* a, void* o,
                                      float* bank_layer, int64_t num_slots,
                                      const int32_t* slot_ids, int32_t B, int32_t T,
                                      int32_t H, int32_t K, int32_t V, int32_t dtype,
                                      int32_t* status, wkvm_stream_t stream) {
  if (!bank_layer || (!slot_ids && B > 0) || num_slots <= 0) return WKVM_ERR_INVALID_ARG;
  RecArgs args{r, w, k, v, kk, a, o, bank_layer, bank_layer, slot_ids, num_slots, nullptr,
               B, T, H, H, K, V, 1.0f, false, status, (cudaStream_t)stream};
  args.overlap = wkvm::g_decode_overlap;
  int rc = wkvm::check_common(args, false);
  if (rc) return rc;
  if (K != V) return WKVM_ERR_SHAPE;
  if (B == 0 || T == 0) return WKVM_OK;
  return wkvm::launch_wkv7<true>(args, dtype);
}

extern "C" int wkvm_fused_recurrent_gated_delta_rule(
    const void* q, const void* k, const void* v, const void* g, const void* beta, void* o,
    const float* h0, float* ht, const int64_t* cu_seqlens, int32_t B, int32_t T, int32_t H,
    int32_t HV, int32_t K, int32_t V, float scale, int32_t use_qk_l2norm, int32_t dtype,
    int32_t* status, wkvm_stream_t stream) {
  RecArgs args{q, k, v, g, beta, beta, o, h0, ht, nullptr, 0, cu_seqlens, B, T, H, HV, K, V,
               scale, use_qk_l2norm != 0, status, (cudaStream_t)stream};
  int rc = wkvm::check_common(args, cu_seqlens != nullptr);
  if (rc) return rc;
  if (HV <= 0 || HV % H != 0) return WKVM_ERR_SHAPE;
  if (B == 0 || (T == 0 && cu_seqlens == nullptr)) {
    if (h0 && ht && h0 != ht) {
      WKVM_CUDA_TRY(cudaMemcpyAsync(ht, h0, (size_t)B * HV * K * V * sizeof(float),
                                    cudaMemcpyDeviceToDevice, (cudaStream_t)stream));
    }
    return WKVM_OK;
  }
  return wkvm::launch_gdn(args, dtype);
}

extern "C" int wkvm_gdn_decode_slots(const void* q, const void* k, const void* v,
                                     const void* g, const void* beta, void* o,
                                     float* bank_layer, int64_t num_slots,
                                     const int32_t* slot_ids, int32_t B, int32_t T, int32_t H,
                                     int32_t HV, int32_t K, int32_t V, float scale,
                                     int32_t use_qk_l2norm, int32_t dtype, int32_t* status,
                                     wkvm_stream_t stream) {
  if (!bank_layer || (!slot_ids && B > 0) || num_slots <= 0) return WKVM_ERR_INVALID_ARG;
  RecArgs args{q, k, v, g, beta, beta, o, bank_layer, bank_layer, slot_ids, num_slots, nullptr,
               B, T, H, HV, K, V, scale, use_qk_l2norm != 0, status, (cudaStream_t)stream};
  int rc = wkvm::check_common(args, false);
  if (rc) return rc;
  if (HV <= 0 || HV % H != 0) return WKVM_ERR_SHAPE;
  if (B == 0 || T == 0) return WKVM_OK;
  return wkvm::launch_gdn(args, dtype);
}

extern "C" int wkvm_set_decode_overlap(int32_t enable) {
  const int prev = wkvm::g_decode_overlap ? 1 : 0;
  wkvm::g_decode_overlap = enable != 0;
  return prev;
}
