// Chunked (WY / UT-transform) prefill of the gated delta rule on the sm_100a
// tensor core (tcgen05.mma kind::tf32, fp32 accumulators in TMEM), K = V = 128.
//
// The gated delta rule is the DPLR recurrence with a per-token scalar decay:
//   h' = e^g h - beta e^g k (k^T h) + beta k v^T
// i.e. D = e^g I, a = k, b = -beta e^g k, and an update key beta k
// (fla/ops/gated_delta_rule/fused_recurrent.py:128-151). With a scalar decay
// every intra-chunk factor is e^(G_t - G_s) for s <= t (G = cumulative g),
// which never exceeds 1, so no scaling reference is needed.
//
// One CTA owns one (sequence, value head, half of V): the 128 x 64 slice of
// the state. Per 64-token chunk (k^ = k normalised when asked, q^ likewise
// times the scale; Gx = G - g; E = diag(-e^g)):
//   [k^; q^] x k^^T                          Gram blocks           (MMA 1)
//   A_ak = [s<t] e^(Gx_t-G_s) beta_s k^_t.k^_s,  A_ab = A_ak E
//   A_qk = [s<=t] e^(G_t-G_s) beta_s q^_t.k^_s, (A_qb = A_qk E)
//   V^T x A_ak^T = (A_ak V)^T                                      (MMA 2)
//   T = (I - A_ab)^-1 (blocked, CUDA cores)
//   (A_ak V)^T T^T = U~^T ,  (k^ e^Gx)^T T^T = W^T                 (MMA S)
//   W' = E W, U' = V + E U~ ; Kh = beta k^ e^(G_C - G)
//   M = diag(e^G_C) + Kh^T W'    P = q^ e^G + A_qk W'               (MMA 3)
//   N = Kh^T U'                  O_intra = A_qk U'
//   S' = M S + N,  O = P S + O_intra                               (MMA 4)
// Initial values (diag(e^G_C), q^ e^G) are written into the accumulators
// before MMA 3, which accumulates onto them; MMA 4 accumulates onto MMA 3's.
// The chunk recurrence is the one fla's chunk_gated_delta_rule implements
// (fla/ops/gated_delta_rule/chunk.py:29-116; reference
// naive_chunk_gated_delta_rule, fla/ops/gated_delta_rule/naive.py:67-161);
// the operand orientation and TMEM dataflow are this file's own.
#include "chunk_common.cuh"

namespace wkvm {
namespace {

using chunkc::RS;
using chunkc::kst4;

constexpr int CH = 64;        // chunk length
constexpr int KD = 128;       // key dim
constexpr int VD = 128;       // value dim
constexpr int VH = 64;        // value columns per CTA
constexpr int NTHREADS = 256;
constexpr uint32_t LBO = 128, SBO64 = 2048, SBO128 = 4096;  // K = 64 / K = 128 tiles
constexpr uint32_t LBO_S = 144, SBO_S = 32 * LBO_S;          // S^T (K = 128), padded
constexpr uint32_t KSTEP = 2 * LBO;
constexpr int QROW = KD * 2 + 16;  // staged q/k row bytes (+16 pad)
constexpr int VROW = VH * 2 + 16;  // staged v half-row bytes

constexpr uint32_t S_Q = 0;
constexpr uint32_t S_K = S_Q + CH * QROW;
constexpr uint32_t S_V = S_K + CH * QROW;
constexpr uint32_t S_KB = S_V + CH * VROW;       // k^ B tile -> inverse scratch -> W'^T
constexpr uint32_t S_VT = S_KB + 16 * SBO64;     // V^T (rows v, K = t); MMA 2 reads 128 rows
constexpr uint32_t S_AK = S_VT + 8 * SBO64;      // A_ak (rows t, K = s)
constexpr uint32_t S_AAB = S_AK + 8 * SBO64;     // A_ab row-major
constexpr uint32_t S_TT = S_AAB + CH * RS * 4;   // T tile
constexpr uint32_t S_UPT = S_TT + 8 * SBO64;     // U'^T (rows v, K = t)
constexpr uint32_t S_ST = S_UPT + 8 * SBO64;     // S^T (rows v, K = k)
constexpr uint32_t SMEM_USED = S_ST + 8 * SBO_S;
constexpr uint32_t SMEM_BYTES = SMEM_USED + 1024;
static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");

constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t T_X1 = 0;     // [k^; q^] (K = 128) -> Kh^T (K = t) | O_intra -> O at 64..127
constexpr uint32_t T_O = 64;
constexpr uint32_t T_D1 = 128;   // Gram -> A_qk in lanes 64..127
constexpr uint32_t T_AKV = 192;  // (A_ak V)^T -> P (with T_AG, 128 columns)
constexpr uint32_t T_AG = 256;   // (k^ e^Gx)^T
constexpr uint32_t T_U = 320;    // U~^T -> N -> S'
constexpr uint32_t T_W = 384;    // W^T -> M (128 columns)

struct GdnArgs {
  const void *q, *k, *v, *g, *beta;
  void* o;
  const float* h_in;
  float* h_out;
  const int32_t* ids;
  int64_t num_slots;
  const int64_t* cu;
  int T, H, HV;
  float scale;
  bool l2norm;
  int* status;
  bool gates_f32 = false;  // g and beta are fp32 (WKVM_GATES_F32)
};

template <typename T>
__device__ __forceinline__ float ld16(const uint8_t* row, int col) {
  return to_f32(reinterpret_cast<const T*>(row)[col]);
}
template <typename T>
__device__ __forceinline__ void ld8(const uint8_t* row, int col, float (&x)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(row + col * 2);
  const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
  for (int i = 0; i < 8; ++i) x[i] = to_f32(e[i]);
}

__device__ __forceinline__ void sync_tc() {
  tc::fence_smem_to_async();
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
}

template <typename Tin>
__global__ void __launch_bounds__(NTHREADS, 1) gdn_chunk_kernel(GdnArgs p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                           ~static_cast<uintptr_t>(1023));
  __shared__ uint64_t mbar;
  __shared__ uint32_t tmem_slot;
  __shared__ float s_g[CH], s_beta[CH], s_G[CH], s_eg[CH], s_kn[CH], s_qn[CH];

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quarter = warp & 3, gh = warp >> 2;
  const int l = quarter * 32 + lane;  // accumulator row / TMEM lane
  const bool lo = l < 64;
  const int r64 = l & 63;
  const int H = p.H, HV = p.HV;
  const int vh = blockIdx.x & 1;
  const int nh = blockIdx.x >> 1;
  const int n = nh / HV, hv = nh - n * HV, hq = hv / (HV / H);

  int64_t row = n;
  if (p.ids) {
    const int32_t id = p.ids[n];
    if (id < 0 || (int64_t)id >= p.num_slots) {
      if (tid == 0) report(p.status, WKVM_ERR_SLOT_RANGE);
      return;
    }
    row = id;
  }
  const int64_t hoff = (row * HV + hv) * (int64_t)(KD * VD);
  int64_t bos, len;
  if (p.cu) {
    bos = p.cu[n];
    len = p.cu[n + 1] - bos;
  } else {
    bos = (int64_t)n * p.T;
    len = p.T;
  }
  const Tin* __restrict__ gq = static_cast<const Tin*>(p.q);
  const Tin* __restrict__ gk = static_cast<const Tin*>(p.k);
  const Tin* __restrict__ gv = static_cast<const Tin*>(p.v);
  Tin* __restrict__ go = static_cast<Tin*>(p.o);

  if (warp == 0) {
    tc::tmem_alloc(&tmem_slot, TMEM_COLS);
    tc::tmem_relinquish();
  }
  if (tid == 0) tc::mbar_init(&mbar, 1);
  for (int e = tid; e < KD * VH; e += NTHREADS) {  // S^T[v][k] = h[k][vh*64 + v]
    const int kk = e >> 6, v = e & 63;
    const float x = p.h_in ? p.h_in[hoff + kk * VD + vh * VH + v] : 0.f;
    *reinterpret_cast<float*>(sm + S_ST + tc::kmajor_off(v, kk, LBO_S, SBO_S)) = x;
  }
  sync_tc();
  const uint32_t tm = tmem_slot;
  const uint32_t tq = tc::tmem_addr(tm, quarter * 32, 0);
  uint32_t phase = 0;
  bool failed = false;
  const int nchunks = (int)((len + CH - 1) / CH);

  auto wait_mma = [&]() -> bool {
    const bool ok = warp != 0 || tc::mbar_wait(&mbar, phase);  // warp 0 polls
    phase ^= 1u;
    const bool any_bad = __syncthreads_or(!ok);
    tc::fence_after_sync();
    if (any_bad && tid == 0) report(p.status, WKVM_ERR_TIMEOUT);
    return !any_bad;
  };

  // q and k rows (16 pieces of 16 B), this CTA's half of the v rows (8 pieces):
  // 2560 pieces, 10 per thread.
  auto stage = [&](int c) {
    const int64_t t0 = bos + (int64_t)c * CH;
    const int64_t rem = len - (int64_t)c * CH;
    const int cl = rem < CH ? (int)rem : CH;
    const uint32_t base = tc::smem_u32(sm);
#pragma unroll
    for (int j = 0; j < 10; ++j) {
      const int e = tid + NTHREADS * j;
      uint32_t off;
      const char* src;
      int t;
      if (e < 2048) {
        const int which = e >> 10, e2 = e & 1023;
        t = e2 >> 4;
        const int piece = e2 & 15;
        off = (which ? S_K : S_Q) + t * QROW + piece * 16;
        src = reinterpret_cast<const char*>(which ? gk : gq) +
              (((t0 + t) * H + hq) * KD) * 2 + piece * 16;
      } else {
        const int e2 = e - 2048;
        t = e2 >> 3;
        const int piece = e2 & 7;
        off = S_V + t * VROW + piece * 16;
        src = reinterpret_cast<const char*>(gv) + (((t0 + t) * HV + hv) * VD + vh * VH) * 2 +
              piece * 16;
      }
      if (t < cl) chunkc::cp_async16(base + off, src);
      else *reinterpret_cast<uint4*>(sm + off) = make_uint4(0, 0, 0, 0);
    }
    chunkc::cp_async_commit();
  };
  if (nchunks > 0) stage(0);
  const uint32_t id64 = tc::idesc_tf32(128, 64), id128 = tc::idesc_tf32(128, 128);

  for (int c = 0; c < nchunks; ++c) {
    const int64_t tok0 = bos + (int64_t)c * CH;
    const int64_t rem = len - (int64_t)c * CH;
    const int clen = rem < CH ? (int)rem : CH;
    const bool last = (c == nchunks - 1);
    chunkc::cp_async_wait_all();
    __syncthreads();

    // ---- per-token scalars (threads 0..63) and V^T (threads 128..255)
    if (tid < CH) {
      const int t = tid;
      const bool valid = t < clen;
      const int64_t gi = (tok0 + t) * HV + hv;
      const float gt = valid ? load_gate<Tin>(p.g, gi, p.gates_f32) : 0.f;
      const float bt = valid ? load_gate<Tin>(p.beta, gi, p.gates_f32) : 0.f;
      float kn = 1.f, qn = 1.f;
      if (p.l2norm) {
        float sk = 0.f, sq = 0.f;
        for (int k8 = 0; k8 < KD; k8 += 8) {
          float xk[8], xq[8];
          ld8<Tin>(sm + S_K + t * QROW, k8, xk);
          ld8<Tin>(sm + S_Q + t * QROW, k8, xq);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            sk = fmaf(xk[i], xk[i], sk);
            sq = fmaf(xq[i], xq[i], sq);
          }
        }
        kn = 1.0f / sqrtf(sk + 1e-6f);
        qn = 1.0f / sqrtf(sq + 1e-6f);
      }
      s_g[t] = gt;
      s_beta[t] = bt;
      s_kn[t] = kn;
      s_qn[t] = qn * p.scale;
      s_eg[t] = __expf(gt);
    } else if (tid >= 128) {
      const int v = tid & 63, t0 = ((tid - 128) >> 6) * 32;
#pragma unroll
      for (int t = t0; t < t0 + 32; t += 4)
        kst4(sm + S_VT, v, t, LBO, SBO64,
             make_float4(ld16<Tin>(sm + S_V + t * VROW, v), ld16<Tin>(sm + S_V + (t + 1) * VROW, v),
                         ld16<Tin>(sm + S_V + (t + 2) * VROW, v),
                         ld16<Tin>(sm + S_V + (t + 3) * VROW, v)));
    }
    __syncthreads();
    if (warp == 0) {  // inclusive cumulative decay over the 64 tokens
      float a = s_g[lane], b = s_g[lane + 32];
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const float ua = __shfl_up_sync(0xffffffffu, a, off);
        const float ub = __shfl_up_sync(0xffffffffu, b, off);
        if (lane >= off) {
          a += ua;
          b += ub;
        }
      }
      b += __shfl_sync(0xffffffffu, a, 31);
      s_G[lane] = a;
      s_G[lane + 32] = b;
    }
    __syncthreads();
    const float GC = s_G[CH - 1];

    // ---- rows: lo lane t: k^ -> TMEM (A of MMA 1) and the B tile row t;
    //            hi lane t: q^ (scaled) -> TMEM. Column half gh of K.
    {
      const int t = r64;
      const uint8_t* src = sm + (lo ? S_K : S_Q) + t * QROW;
      const float f = lo ? s_kn[t] : s_qn[t];
#pragma unroll 1
      for (int h2 = 0; h2 < 2; ++h2) {
        const int k0 = gh * 64 + h2 * 32;
        float x[32];
#pragma unroll
        for (int k8 = 0; k8 < 32; k8 += 8) {
          float y[8];
          ld8<Tin>(src, k0 + k8, y);
#pragma unroll
          for (int i = 0; i < 8; ++i) x[k8 + i] = y[i] * f;
        }
        tc::tmem_st32(tq + T_X1 + k0, x);
        if (lo) {
#pragma unroll
          for (int i = 0; i < 32; i += 4)
            kst4(sm + S_KB, t, k0 + i, LBO, SBO128, make_float4(x[i], x[i + 1], x[i + 2], x[i + 3]));
        }
      }
      tc::tmem_st_wait();
    }
    sync_tc();

    // ---- MMA 1: [k^; q^] x k^^T -> T_D1 (Gram blocks)
    if (tid == 0) {
      const uint64_t b0 = tc::smem_desc(tc::smem_u32(sm + S_KB), LBO, SBO128);
#pragma unroll
      for (int kk = 0; kk < KD / 8; ++kk)
        tc::mma_tf32_ta(tm + T_D1, tm + T_X1 + kk * 8, tc::desc_add(b0, kk * KSTEP), id64, kk > 0);
      tc::mma_commit(&mbar);
    }
    if (!wait_mma()) { failed = true; break; }

    // ---- gates and masks: lo rows -> A_ak tile and A_ab; hi rows -> A_qk in place
    {
      const int t = r64, s0 = gh * 32;
      float x[32];
      tc::tmem_ld32(tq + T_D1 + s0, x);
      if (lo) {
        const float gx = s_G[t] - s_g[t];
        float ab[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int s = s0 + i;
          const float v = (s < t) ? __expf(gx - s_G[s]) * s_beta[s] * x[i] : 0.f;
          x[i] = v;
          ab[i] = -v * s_eg[s];
        }
#pragma unroll
        for (int i = 0; i < 32; i += 4) {
          kst4(sm + S_AK, t, s0 + i, LBO, SBO64, make_float4(x[i], x[i + 1], x[i + 2], x[i + 3]));
          *reinterpret_cast<float4*>(reinterpret_cast<float*>(sm + S_AAB) + t * RS + s0 + i) =
              make_float4(ab[i], ab[i + 1], ab[i + 2], ab[i + 3]);
        }
      } else {
        const float gt = s_G[t];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int s = s0 + i;
          x[i] = (s <= t) ? __expf(gt - s_G[s]) * s_beta[s] * x[i] : 0.f;
        }
        tc::tmem_st32(tq + T_D1 + s0, x);
      }
      tc::tmem_st_wait();
    }
    sync_tc();

    // ---- MMA 2: V^T x A_ak^T -> T_AKV lanes v (rows 64..127 of A read into
    //      the A_ak tile and give unused rows)
    if (tid == 0) {
      const uint64_t a0 = tc::smem_desc(tc::smem_u32(sm + S_VT), LBO, SBO64);
      const uint64_t b0 = tc::smem_desc(tc::smem_u32(sm + S_AK), LBO, SBO64);
#pragma unroll
      for (int kk = 0; kk < CH / 8; ++kk)
        tc::mma_tf32(tm + T_AKV, tc::desc_add(a0, kk * KSTEP), tc::desc_add(b0, kk * KSTEP), id64,
                     kk > 0);
      tc::mma_commit(&mbar);
    }
    if (!wait_mma()) { failed = true; break; }

    // ---- columns (lane = key k, tokens of half gh): Kh^T -> T_X1,
    //      (k^ e^Gx)^T -> T_AG
    {
      const int kk = l, t0 = gh * 32;
      float x[32], y[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int t = t0 + i;
        const float kh = ld16<Tin>(sm + S_K + t * QROW, kk) * s_kn[t];
        x[i] = s_beta[t] * kh * __expf(GC - s_G[t]);
        y[i] = kh * __expf(s_G[t] - s_g[t]);
      }
      tc::tmem_st32(tq + T_X1 + t0, x);
      tc::tmem_st32(tq + T_AG + t0, y);
      tc::tmem_st_wait();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();

    // ---- T = (I - A_ab)^-1 (the k^ B tile is spent: its region is scratch)
    chunkc::tri_inverse64(reinterpret_cast<const float*>(sm + S_AAB),
                          reinterpret_cast<float*>(sm + S_KB), sm + S_TT, tid);
    sync_tc();

    // ---- MMA S: (A_ak V)^T T^T -> U~^T ; (k^ e^Gx)^T T^T -> W^T
    if (tid == 0) {
      const uint64_t b0 = tc::smem_desc(tc::smem_u32(sm + S_TT), LBO, SBO64);
#pragma unroll
      for (int kk = 0; kk < CH / 8; ++kk)
        tc::mma_tf32_ta(tm + T_U, tm + T_AKV + kk * 8, tc::desc_add(b0, kk * KSTEP), id64, kk > 0);
#pragma unroll
      for (int kk = 0; kk < CH / 8; ++kk)
        tc::mma_tf32_ta(tm + T_W, tm + T_AG + kk * 8, tc::desc_add(b0, kk * KSTEP), id64, kk > 0);
      tc::mma_commit(&mbar);
    }
    if (!wait_mma()) { failed = true; break; }

    // ---- W'^T = W^T E -> B tile (rows j); U'^T = V^T + U~^T E -> B tile (rows v)
    {
      const int t0 = gh * 32;
      float x[32];
      tc::tmem_ld32(tq + T_W + t0, x);
#pragma unroll
      for (int i = 0; i < 32; i += 4)
        kst4(sm + S_KB, l, t0 + i, LBO, SBO64,
             make_float4(-s_eg[t0 + i] * x[i], -s_eg[t0 + i + 1] * x[i + 1],
                         -s_eg[t0 + i + 2] * x[i + 2], -s_eg[t0 + i + 3] * x[i + 3]));
      tc::tmem_ld32(tq + T_U + t0, x);
      if (lo) {
        const int v = l;
        float u[4];
#pragma unroll
        for (int i = 0; i < 32; i += 4) {
#pragma unroll
          for (int j = 0; j < 4; ++j)
            u[j] = ld16<Tin>(sm + S_V + (t0 + i + j) * VROW, v) - s_eg[t0 + i + j] * x[i + j];
          kst4(sm + S_UPT, v, t0 + i, LBO, SBO64, make_float4(u[0], u[1], u[2], u[3]));
        }
      }
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    // accumulator initial values: diag(e^G_C) under M, q^ e^G under P
    {
      const float egc = __expf(GC);
      float x[32];
#pragma unroll 1
      for (int h2 = 0; h2 < 2; ++h2) {
        const int c0 = gh * 64 + h2 * 32;
#pragma unroll
        for (int i = 0; i < 32; ++i) x[i] = (c0 + i == l) ? egc : 0.f;
        tc::tmem_st32(tq + T_W + c0, x);
        if (!lo) {
          const int t = r64;
          const float f = s_qn[t] * __expf(s_G[t]);
#pragma unroll
          for (int k8 = 0; k8 < 32; k8 += 8) {
            float y[8];
            ld8<Tin>(sm + S_Q + t * QROW, c0 + k8, y);
#pragma unroll
            for (int i = 0; i < 8; ++i) x[k8 + i] = y[i] * f;
          }
          tc::tmem_st32(tq + T_AKV + c0, x);
        }
      }
      tc::tmem_st_wait();
    }
    sync_tc();

    // ---- MMA 3: M += Kh^T W' ; N = Kh^T U' ; P += A_qk W' ; O_intra = A_qk U'
    if (tid == 0) {
      const uint64_t w0 = tc::smem_desc(tc::smem_u32(sm + S_KB), LBO, SBO64);
      const uint64_t u0 = tc::smem_desc(tc::smem_u32(sm + S_UPT), LBO, SBO64);
#pragma unroll
      for (int kk = 0; kk < CH / 8; ++kk) {
        const uint64_t wd = tc::desc_add(w0, kk * KSTEP);
        const uint64_t ud = tc::desc_add(u0, kk * KSTEP);
        tc::mma_tf32_ta(tm + T_W, tm + T_X1 + kk * 8, wd, id128, true);
        tc::mma_tf32_ta(tm + T_U, tm + T_X1 + kk * 8, ud, id64, kk > 0);
        tc::mma_tf32_ta(tm + T_AKV, tm + T_D1 + kk * 8, wd, id128, true);
        tc::mma_tf32_ta(tm + T_O, tm + T_D1 + kk * 8, ud, id64, kk > 0);
      }
      tc::mma_commit(&mbar);
    }
    // staged q/k/v are spent: stage the next chunk (after MMA 3 is issued, so
    // that the issuing thread does not queue behind its share of the copies)
    if (c + 1 < nchunks) stage(c + 1);
    if (!wait_mma()) { failed = true; break; }

    // ---- MMA 4: S' = M S + N ; O = P S + O_intra
    if (tid == 0) {
      const uint64_t s0 = tc::smem_desc(tc::smem_u32(sm + S_ST), LBO_S, SBO_S);
#pragma unroll
      for (int kk = 0; kk < KD / 8; ++kk) {
        const uint64_t sd = tc::desc_add(s0, kk * 2 * LBO_S);
        tc::mma_tf32_ta(tm + T_U, tm + T_W + kk * 8, sd, id64, true);
        tc::mma_tf32_ta(tm + T_O, tm + T_AKV + kk * 8, sd, id64, true);
      }
      tc::mma_commit(&mbar);
    }
    if (!wait_mma()) { failed = true; break; }

    {
      const int v0 = gh * 32;
      float x[32];
      tc::tmem_ld32(tq + T_U + v0, x);  // S'[k = l][v0 + i]
#pragma unroll
      for (int i = 0; i < 32; ++i)
        *reinterpret_cast<float*>(sm + S_ST + tc::kmajor_off(v0 + i, l, LBO_S, SBO_S)) = x[i];
      if (last && p.h_out) {
        float* dst = p.h_out + hoff + l * VD + vh * VH + v0;
#pragma unroll
        for (int i = 0; i < 32; i += 4)
          st_stream_f4(dst + i, make_float4(x[i], x[i + 1], x[i + 2], x[i + 3]));
      }
      tc::tmem_ld32(tq + T_O + v0, x);  // O[t = l - 64][v0 + i]
      if (!lo) {
        const int t = r64;
        if (t < clen) {
          Tin* dst = go + ((tok0 + t) * HV + hv) * VD + vh * VH + v0;
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            uint4 u;
            Tin* e = reinterpret_cast<Tin*>(&u);
#pragma unroll
            for (int j = 0; j < 8; ++j) e[j] = from_f32<Tin>(x[i + j]);
            *reinterpret_cast<uint4*>(dst + i) = u;
          }
        }
      }
    }
    sync_tc();
  }

  chunkc::cp_async_wait_all();
  if (failed) {
    tc::mbar_wait(&mbar, phase ^ 1u);
  } else if (nchunks == 0 && p.h_out && p.h_out != p.h_in) {
    for (int e = tid; e < KD * VH; e += NTHREADS) {
      const int kk = e >> 6, v = e & 63;
      const int64_t i = hoff + kk * VD + vh * VH + v;
      p.h_out[i] = p.h_in ? p.h_in[i] : 0.f;
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tm, TMEM_COLS);
}

template <typename Tin>
int launch_gdn_chunk(const GdnArgs& a, int nblocks, cudaStream_t stream) {
  auto k = gdn_chunk_kernel<Tin>;
  WKVM_CUDA_TRY(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
  k<<<nblocks, NTHREADS, SMEM_BYTES, stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? WKVM_OK : WKVM_ERR_CUDA;
}

bool al16(const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; }

bool gdn_chunk_ok(int K, int V, int dtype, const void* q, const void* k, const void* v,
                  const void* o) {
  const int act = dtype & ~WKVM_GATES_F32;
  return K == KD && V == VD && (act == WKVM_DTYPE_BF16 || act == WKVM_DTYPE_F16) &&
         al16(q) && al16(k) && al16(v) && al16(o);
}

int run_gdn_chunk(GdnArgs a, int nseq, int dtype, cudaStream_t stream) {
  const int nblocks = nseq * a.HV * 2;
  a.gates_f32 = (dtype & WKVM_GATES_F32) != 0;
  if ((dtype & ~WKVM_GATES_F32) == WKVM_DTYPE_BF16)
    return launch_gdn_chunk<__nv_bfloat16>(a, nblocks, stream);
  return launch_gdn_chunk<__half>(a, nblocks, stream);
}

}  // namespace

int gdn_two_phase(const void* q, const void* k, const void* v, const void* g, const void* beta,
                  void* o, const float* h_in, float* h_out, bool slots, const int32_t* ids,
                  int64_t num_slots, const int64_t* cu, int nseq, int T, int H, int HV,
                  float scale, bool l2norm, int dtype, void* workspace, int64_t ws_bytes,
                  int* status, cudaStream_t stream);

}  // namespace wkvm

extern "C" int wkvm_fused_recurrent_gated_delta_rule(
    const void*, const void*, const void*, const void*, const void*, void*, const float*, float*,
    const int64_t*, int32_t, int32_t, int32_t, int32_t, int32_t, int32_t, float, int32_t, int32_t,
    int32_t*, wkvm_stream_t);
extern "C" int wkvm_gdn_decode_slots(const void*, const void*, const void*, const void*,
                                     const void*, void*, float*, int64_t, const int32_t*,
                                     int32_t, int32_t, int32_t, int32_t, int32_t, int32_t, float,
                                     int32_t, int32_t, int32_t*, wkvm_stream_t);

extern "C" int wkvm_chunk_gated_delta_rule(const void* q, const void* k, const void* v,
                                           const void* g, const void* beta, void* o,
                                           const float* h0, float* ht, const int64_t* cu_seqlens,
                                           int32_t B, int32_t T, int32_t H, int32_t HV, int32_t K,
                                           int32_t V, float scale, int32_t use_qk_l2norm,
                                           int32_t dtype, void* workspace,
                                           int64_t workspace_bytes, int32_t* status,
                                           wkvm_stream_t stream) {
  if (!wkvm::gdn_chunk_ok(K, V, dtype, q, k, v, o))
    return wkvm_fused_recurrent_gated_delta_rule(q, k, v, g, beta, o, h0, ht, cu_seqlens, B, T, H,
                                                 HV, K, V, scale, use_qk_l2norm, dtype, status,
                                                 stream);
  if (B < 0 || T < 0 || H <= 0 || HV <= 0 || HV % H) return WKVM_ERR_INVALID_ARG;
  if (B == 0) return WKVM_OK;
  if (!g || !beta) return WKVM_ERR_INVALID_ARG;
  if ((h0 && !wkvm::al16(h0)) || (ht && !wkvm::al16(ht))) return WKVM_ERR_ALIGN;
  if (workspace) {
    const int r = wkvm::gdn_two_phase(q, k, v, g, beta, o, h0, ht, false, nullptr, 0, cu_seqlens,
                                      B, T, H, HV, scale, use_qk_l2norm != 0, dtype, workspace,
                                      workspace_bytes, status, (cudaStream_t)stream);
    if (r != WKVM_ERR_UNSUPPORTED) return r;
  }
  wkvm::GdnArgs a{q, k, v, g, beta, o, h0, ht, nullptr, 0, cu_seqlens, T, H, HV, scale,
                  use_qk_l2norm != 0, status};
  return wkvm::run_gdn_chunk(a, B, dtype, (cudaStream_t)stream);
}

extern "C" int wkvm_gdn_prefill_slots(const void* q, const void* k, const void* v, const void* g,
                                      const void* beta, void* o, float* bank_layer,
                                      int64_t num_slots, const int32_t* slot_ids,
                                      const int64_t* cu_seqlens, int32_t B, int32_t T, int32_t H,
                                      int32_t HV, int32_t K, int32_t V, float scale,
                                      int32_t use_qk_l2norm, int32_t dtype, void* workspace,
                                      int64_t workspace_bytes, int32_t* status,
                                      wkvm_stream_t stream) {
  if (!bank_layer || num_slots <= 0 || (B > 0 && !slot_ids)) return WKVM_ERR_INVALID_ARG;
  if (!wkvm::gdn_chunk_ok(K, V, dtype, q, k, v, o)) {
    if (cu_seqlens) return WKVM_ERR_UNSUPPORTED;
    return wkvm_gdn_decode_slots(q, k, v, g, beta, o, bank_layer, num_slots, slot_ids, B, T, H,
                                 HV, K, V, scale, use_qk_l2norm, dtype, status, stream);
  }
  if (B < 0 || T < 0 || H <= 0 || HV <= 0 || HV % H) return WKVM_ERR_INVALID_ARG;
  if (B == 0) return WKVM_OK;
  if (!g || !beta) return WKVM_ERR_INVALID_ARG;
  if (!wkvm::al16(bank_layer)) return WKVM_ERR_ALIGN;
  if (workspace) {
    const int r = wkvm::gdn_two_phase(q, k, v, g, beta, o, bank_layer, bank_layer, true, slot_ids,
                                      num_slots, cu_seqlens, B, T, H, HV, scale,
                                      use_qk_l2norm != 0, dtype, workspace, workspace_bytes,
                                      status, (cudaStream_t)stream);
    if (r != WKVM_ERR_UNSUPPORTED) return r;
  }
  wkvm::GdnArgs a{q, k, v, g, beta, o, bank_layer, bank_layer, slot_ids, num_slots, cu_seqlens,
                  T, H, HV, scale, use_qk_l2norm != 0, status};
  return wkvm::run_gdn_chunk(a, B, dtype, (cudaStream_t)stream);
}
