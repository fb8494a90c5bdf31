// Chunked (WY / UT-transform) prefill of the RWKV-7 DPLR recurrence on the
// sm_100a tensor core (tcgen05.mma kind::tf32, fp32 accumulators in TMEM).
//
// One CTA owns one (sequence, head) and walks its 64-token chunks in order,
// keeping every intermediate in shared memory and TMEM; HBM sees only the
// bf16 inputs, the bf16 outputs and the fp32 state once in and once out.
//
// Per chunk (rows t, s = tokens, k, j = key index, v = value index; G = the
// inclusive cumulative log-decay, Gx = G - w the exclusive one, g0 = G at the
// chunk midpoint as a scaling reference, C = the last row):
//   [a e^(Gx-g0); r e^(G-g0)] x [k e^(g0-G); b e^(g0-G)]^T
//        -> A_ak (s<t), A_ab (s<t), A_qk (s<=t), A_qb (s<=t)         (MMA 1)
//   A_ak V                                                            (MMA 2)
//   (I - A_ab) [W | U~] = [a e^Gx | A_ak V]     forward substitution, fp32
//   [A_qb; Bh^T] x [W | U~] + [A_qk; Kh^T] x V                       (MMA 3)
//        with Kh = k e^(G_C - G), Bh = b e^(G_C - G)
//   P = r e^G + A_qb W,  M = diag(e^G_C) + Bh^T W
//   [O; S'] = [P; M] x S + [A_qk V + A_qb U~; Kh^T V + Bh^T U~]       (MMA 4)
// MMA 4 accumulates onto the TMEM columns MMA 3 left, so the chunk's
// output and next state come out of one instruction group.
//
// Algebra and operand orientation are this file's own; the chunk recurrence
// is the one fla's chunk_dplr_delta_rule implements
// (fla/ops/generalized_delta_rule/dplr/chunk.py:33-135, reference
// dplr_chunkwise in .../dplr/naive.py:41-101). tf32 operands keep the result
// within 2e-3 of the fp32 recurrence after 4096 tokens; bf16 operands do not.
#include "tcgen05.cuh"

namespace wkvm {
namespace {

constexpr int CH = 64;             // chunk length
constexpr int HD = 64;             // head dim (K == V)
constexpr int NTHREADS = 128;      // one thread per TMEM lane
constexpr uint32_t LBO = 128;      // K-adjacent core matrices
constexpr uint32_t SBO = 2048;     // 8-row groups of a 64-wide K tile
constexpr uint32_t TILE = 16384;   // 64 x 64 fp32
constexpr uint32_t KSTEP = 2 * LBO;  // 8 tf32 (32 bytes) of K per MMA
// shared-memory regions (bytes), reused across a chunk as noted
constexpr uint32_t R1 = 0;               // [a~; r~] -> {A_ab, A_ak V} row-major -> [P; M]
constexpr uint32_t R2 = R1 + 2 * TILE;   // [k~; b~] -> [W^T; U~^T]
constexpr uint32_t R3 = R2 + 2 * TILE;   // G scratch | [A_ak][A_qk][Kh^T]
constexpr uint32_t R4 = R3 + 3 * TILE;   // [A_qb][Bh^T]
constexpr uint32_t R5 = R4 + 2 * TILE;   // V^T
constexpr uint32_t R6 = R5 + TILE;       // S^T (the running state)
constexpr uint32_t R7 = R6 + TILE;       // a e^Gx row-major
constexpr uint32_t R8 = R7 + TILE;       // r e^G row-major
constexpr uint32_t SMEM_USED = R8 + TILE;
constexpr uint32_t SMEM_BYTES = SMEM_USED + 1024;  // + alignment slack
constexpr uint32_t TMEM_COLS = 256;

struct ChunkArgs {
  const void *p0, *p1, *p2, *p3, *p4, *p5;  // r, w, k, v, (kk | a), (a_gate | b)
  void* o;
  const float* h_in;
  float* h_out;
  const int32_t* ids;
  int64_t num_slots;
  const int64_t* cu;
  int T, H;
  float scale;
  int* status;
};

__device__ __forceinline__ void kst(uint8_t* tile, int row, int k, float x) {
  *reinterpret_cast<float*>(tile + tc::kmajor_off(row, k, LBO, SBO)) = x;
}
__device__ __forceinline__ void kst4(uint8_t* tile, int row, int k, float4 x) {
  *reinterpret_cast<float4*>(tile + tc::kmajor_off(row, k, LBO, SBO)) = x;
}

template <typename T>
__device__ __forceinline__ void store_row32(T* dst, const float (&v)[32]) {
#pragma unroll
  for (int i = 0; i < 32; ++i) dst[i] = from_f32<T>(v[i]);
}
template <>
__device__ __forceinline__ void store_row32<__nv_bfloat16>(__nv_bfloat16* dst, const float (&v)[32]) {
#pragma unroll
  for (int i = 0; i < 32; i += 8) {
    uint4 u;
    __nv_bfloat162 b0 = __floats2bfloat162_rn(v[i + 0], v[i + 1]);
    __nv_bfloat162 b1 = __floats2bfloat162_rn(v[i + 2], v[i + 3]);
    __nv_bfloat162 b2 = __floats2bfloat162_rn(v[i + 4], v[i + 5]);
    __nv_bfloat162 b3 = __floats2bfloat162_rn(v[i + 6], v[i + 7]);
    u.x = *reinterpret_cast<uint32_t*>(&b0);
    u.y = *reinterpret_cast<uint32_t*>(&b1);
    u.z = *reinterpret_cast<uint32_t*>(&b2);
    u.w = *reinterpret_cast<uint32_t*>(&b3);
    *reinterpret_cast<uint4*>(dst + i) = u;
  }
}

__device__ __forceinline__ void sync_tc() {
  tc::fence_smem_to_async();
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
}

template <typename Tin, bool MUL>
__global__ void __launch_bounds__(NTHREADS, 1) dplr_chunk_kernel(ChunkArgs p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                           ~static_cast<uintptr_t>(1023));
  __shared__ uint64_t mbar;
  __shared__ uint32_t tmem_slot;
  __shared__ float s_gc[HD];

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nh = blockIdx.x;
  const int n = nh / p.H;
  const int hh = nh - n * p.H;
  const int H = p.H;

  int64_t row = n;
  if (p.ids) {
    const int32_t id = p.ids[n];
    if (id < 0 || (int64_t)id >= p.num_slots) {
      if (tid == 0) report(p.status, WKVM_ERR_SLOT_RANGE);
      return;
    }
    row = id;
  }
  const int64_t hoff = (row * H + hh) * (int64_t)(HD * HD);
  int64_t bos, len;
  if (p.cu) {
    bos = p.cu[n];
    len = p.cu[n + 1] - bos;
  } else {
    bos = (int64_t)n * p.T;
    len = p.T;
  }
  const Tin* __restrict__ gr = static_cast<const Tin*>(p.p0);
  const Tin* __restrict__ gw = static_cast<const Tin*>(p.p1);
  const Tin* __restrict__ gk = static_cast<const Tin*>(p.p2);
  const Tin* __restrict__ gv = static_cast<const Tin*>(p.p3);
  const Tin* __restrict__ g5 = static_cast<const Tin*>(p.p4);
  const Tin* __restrict__ g6 = static_cast<const Tin*>(p.p5);
  Tin* __restrict__ go = static_cast<Tin*>(p.o);

  if (warp == 0) {
    tc::tmem_alloc(&tmem_slot, TMEM_COLS);
    tc::tmem_relinquish();
  }
  if (tid == 0) tc::mbar_init(&mbar, 1);
  // S^T[v][k] = h[k][v]
  for (int e = tid; e < HD * HD; e += NTHREADS) {
    const int k = e >> 6, v = e & 63;
    kst(sm + R6, v, k, p.h_in ? p.h_in[hoff + e] : 0.f);
  }
  sync_tc();
  const uint32_t tm = tmem_slot;
  uint32_t phase = 0;
  bool failed = false;
  const int nchunks = (int)((len + CH - 1) / CH);
  float* G = reinterpret_cast<float*>(sm + R3);
  float* Arow = reinterpret_cast<float*>(sm + R1);
  float* AkV = reinterpret_cast<float*>(sm + R1 + TILE);
  float* ag = reinterpret_cast<float*>(sm + R7);
  float* rg = reinterpret_cast<float*>(sm + R8);
  const int drow = warp * 32 + lane;  // TMEM lane == accumulator row of this thread

  auto wait_mma = [&]() -> bool {
    bool ok = tc::mbar_wait(&mbar, phase);
    phase ^= 1u;
    const bool any_bad = __syncthreads_or(!ok);
    tc::fence_after_sync();
    if (any_bad && tid == 0) report(p.status, WKVM_ERR_TIMEOUT);
    return !any_bad;
  };

  for (int c = 0; c < nchunks && !failed; ++c) {
    const int64_t tok0 = bos + (int64_t)c * CH;
    const int64_t rem = len - (int64_t)c * CH;
    const int clen = rem < CH ? (int)rem : CH;
    const bool last = (c == nchunks - 1);

    // ---- cumulative log-decay G[t][k] (two halves of 32 tokens, then joined)
    {
      const int k = tid & 63, half = tid >> 6;
      float g = 0.f;
      for (int i = 0; i < 32; ++i) {
        const int t = half * 32 + i;
        const float wt = (t < clen) ? to_f32(gw[((tok0 + t) * H + hh) * HD + k]) : 0.f;
        g += wt;
        G[t * 64 + k] = g;
      }
    }
    __syncthreads();
    if (tid >= 64) {
      const int k = tid - 64;
      const float base = G[31 * 64 + k];
      for (int t = 32; t < 64; ++t) G[t * 64 + k] += base;
    }
    __syncthreads();

    // ---- elementwise operands
    if (tid < 64) {
      s_gc[tid] = expf(G[63 * 64 + tid]);
      // exp(+-(G - G_mid)) must stay finite in fp32 (e^88); RWKV-7's decay
      // (w >= -0.61 per token) keeps the span under 20.
      const float span = fmaxf(fabsf(G[tid] - G[31 * 64 + tid]), fabsf(G[63 * 64 + tid] - G[31 * 64 + tid]));
      if (span > 80.f) report(p.status, WKVM_ERR_UNSUPPORTED);
    }
#pragma unroll 2
    for (int i = 0; i < (CH * HD) / NTHREADS; ++i) {
      const int e = i * NTHREADS + tid;
      const int t = e >> 6, k = e & 63;
      float rr = 0.f, wt = 0.f, kv = 0.f, vv = 0.f, aa = 0.f, bb = 0.f;
      if (t < clen) {
        const int64_t gi = ((tok0 + t) * H + hh) * HD + k;
        rr = to_f32(gr[gi]) * p.scale;
        wt = to_f32(gw[gi]);
        kv = to_f32(gk[gi]);
        vv = to_f32(gv[gi]);
        const float x5 = to_f32(g5[gi]);
        const float x6 = to_f32(g6[gi]);
        aa = MUL ? -x5 : x5;
        bb = MUL ? x5 * x6 : x6;
      }
      const float gt = G[t * 64 + k];
      const float gx = gt - wt;
      const float ref = G[31 * 64 + k];
      const float gc = G[63 * 64 + k];
      kst(sm + R1, t, k, aa * expf(gx - ref));
      kst(sm + R1, 64 + t, k, rr * expf(gt - ref));
      const float einv = expf(ref - gt);
      kst(sm + R2, t, k, kv * einv);
      kst(sm + R2, 64 + t, k, bb * einv);
      ag[t * 64 + k] = aa * expf(gx);
      rg[t * 64 + k] = rr * expf(gt);
      const float ec = expf(gc - gt);
      kst(sm + R3 + 2 * TILE, k, t, kv * ec);  // Kh^T
      kst(sm + R4 + TILE, k, t, bb * ec);      // Bh^T
      kst(sm + R5, k, t, vv);                  // V^T
    }
    sync_tc();

    // ---- MMA 1: [a~; r~] x [k~; b~]^T -> TMEM cols [0, 128)
    if (tid == 0) {
      const uint32_t id = tc::idesc_tf32(128, 128);
      const uint32_t a0 = tc::smem_u32(sm + R1), b0 = tc::smem_u32(sm + R2);
      for (int kk = 0; kk < HD / 8; ++kk)
        tc::mma_tf32(tm, tc::smem_desc(a0 + kk * KSTEP, LBO, SBO),
                     tc::smem_desc(b0 + kk * KSTEP, LBO, SBO), id, kk > 0);
      tc::mma_commit(&mbar);
    }
    if (!wait_mma()) { failed = true; break; }

    // ---- split into the four masked intra-chunk matrices
#pragma unroll 1
    for (int cb = 0; cb < 4; ++cb) {
      float vals[32];
      tc::tmem_ld32(tc::tmem_addr(tm, warp * 32, cb * 32), vals);
      const bool kcols = cb < 2;
      if (drow < 64) {
        const int t = drow;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int s = (cb & 1) * 32 + i;
          const float x = (s < t) ? vals[i] : 0.f;
          if (kcols) kst(sm + R3, t, s, x);   // A_ak
          else Arow[t * 64 + s] = x;          // A_ab (row-major, for the solve)
        }
      } else {
        const int t = drow - 64;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int s = (cb & 1) * 32 + i;
          const float x = (s <= t) ? vals[i] : 0.f;
          if (kcols) kst(sm + R3 + TILE, t, s, x);  // A_qk
          else kst(sm + R4, t, s, x);               // A_qb
        }
      }
    }
    sync_tc();

    // ---- MMA 2: [A_ak; A_qk] x V -> TMEM cols [128, 192) (top half used)
    if (tid == 0) {
      const uint32_t id = tc::idesc_tf32(128, 64);
      const uint32_t a0 = tc::smem_u32(sm + R3), b0 = tc::smem_u32(sm + R5);
      for (int kk = 0; kk < CH / 8; ++kk)
        tc::mma_tf32(tm + 128, tc::smem_desc(a0 + kk * KSTEP, LBO, SBO),
                     tc::smem_desc(b0 + kk * KSTEP, LBO, SBO), id, kk > 0);
      tc::mma_commit(&mbar);
    }
    if (!wait_mma()) { failed = true; break; }
    if (warp < 2) {
#pragma unroll 1
      for (int cb = 0; cb < 2; ++cb) {
        float vals[32];
        tc::tmem_ld32(tc::tmem_addr(tm, warp * 32, 128 + cb * 32), vals);
#pragma unroll
        for (int i = 0; i < 32; ++i) AkV[drow * 64 + cb * 32 + i] = vals[i];
      }
    }
    tc::fence_before_sync();
    __syncthreads();

    // ---- forward substitution: (I - A_ab) y = rhs, one column per thread
    {
      const int col = tid & 63;
      const float* rhs = (tid < 64) ? ag : AkV;
      float y[CH];
#pragma unroll
      for (int t = 0; t < CH; ++t) {
        float a0 = rhs[t * 64 + col], a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
        for (int s = 0; s + 4 <= t; s += 4) {
          const float4 av = *reinterpret_cast<const float4*>(&Arow[t * 64 + s]);
          a0 = fmaf(av.x, y[s], a0);
          a1 = fmaf(av.y, y[s + 1], a1);
          a2 = fmaf(av.z, y[s + 2], a2);
          a3 = fmaf(av.w, y[s + 3], a3);
        }
#pragma unroll
        for (int s = t & ~3; s < t; ++s) a0 = fmaf(Arow[t * 64 + s], y[s], a0);
        y[t] = (a0 + a1) + (a2 + a3);
      }
      uint8_t* dst = sm + R2 + (tid < 64 ? 0 : TILE);  // W^T | U~^T, row = column index
#pragma unroll
      for (int t = 0; t < CH; t += 4) kst4(dst, col, t, make_float4(y[t], y[t + 1], y[t + 2], y[t + 3]));
    }
    sync_tc();

    // ---- MMA 3: [A_qb; Bh^T] x [W | U~] -> cols [0,128); += [A_qk; Kh^T] x V -> cols [64,128)
    if (tid == 0) {
      const uint32_t id128 = tc::idesc_tf32(128, 128), id64 = tc::idesc_tf32(128, 64);
      const uint32_t a0 = tc::smem_u32(sm + R4), b0 = tc::smem_u32(sm + R2);
      for (int kk = 0; kk < CH / 8; ++kk)
        tc::mma_tf32(tm, tc::smem_desc(a0 + kk * KSTEP, LBO, SBO),
                     tc::smem_desc(b0 + kk * KSTEP, LBO, SBO), id128, kk > 0);
      const uint32_t a1 = tc::smem_u32(sm + R3 + TILE), b1 = tc::smem_u32(sm + R5);
      for (int kk = 0; kk < CH / 8; ++kk)
        tc::mma_tf32(tm + 64, tc::smem_desc(a1 + kk * KSTEP, LBO, SBO),
                     tc::smem_desc(b1 + kk * KSTEP, LBO, SBO), id64, true);
      tc::mma_commit(&mbar);
    }
    if (!wait_mma()) { failed = true; break; }

    // ---- P = r e^G + A_qb W ; M = diag(e^G_C) + Bh^T W  -> [P; M] in R1
#pragma unroll 1
    for (int cb = 0; cb < 2; ++cb) {
      float vals[32];
      tc::tmem_ld32(tc::tmem_addr(tm, warp * 32, cb * 32), vals);
      if (drow < 64) {
        const int t = drow;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int j = cb * 32 + i;
          kst(sm + R1, t, j, rg[t * 64 + j] + vals[i]);
        }
      } else {
        const int kr = drow - 64;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int j = cb * 32 + i;
          kst(sm + R1 + TILE, kr, j, vals[i] + (j == kr ? s_gc[kr] : 0.f));
        }
      }
    }
    sync_tc();

    // ---- MMA 4: [O; S'] = [P; M] x S + [O_intra; N] (accumulate on cols [64,128))
    if (tid == 0) {
      const uint32_t id = tc::idesc_tf32(128, 64);
      const uint32_t a0 = tc::smem_u32(sm + R1), b0 = tc::smem_u32(sm + R6);
      for (int kk = 0; kk < HD / 8; ++kk)
        tc::mma_tf32(tm + 64, tc::smem_desc(a0 + kk * KSTEP, LBO, SBO),
                     tc::smem_desc(b0 + kk * KSTEP, LBO, SBO), id, true);
      tc::mma_commit(&mbar);
    }
    if (!wait_mma()) { failed = true; break; }

#pragma unroll 1
    for (int cb = 0; cb < 2; ++cb) {
      float vals[32];
      tc::tmem_ld32(tc::tmem_addr(tm, warp * 32, 64 + cb * 32), vals);
      if (drow < 64) {
        const int t = drow;
        if (t < clen) store_row32(go + ((tok0 + t) * H + hh) * HD + cb * 32, vals);
      } else {
        const int kr = drow - 64;
#pragma unroll
        for (int i = 0; i < 32; ++i) kst(sm + R6, cb * 32 + i, kr, vals[i]);
        if (last && p.h_out) {
          float* dst = p.h_out + hoff + kr * 64 + cb * 32;
#pragma unroll
          for (int i = 0; i < 32; i += 4)
            st_stream_f4(dst + i, make_float4(vals[i], vals[i + 1], vals[i + 2], vals[i + 3]));
        }
      }
    }
    sync_tc();
  }

  if (failed) {
    // an MMA group may still be running: give it a bounded chance to land
    tc::mbar_wait(&mbar, phase ^ 1u);
  } else if (nchunks == 0 && p.h_out && p.h_out != p.h_in) {
    for (int e = tid; e < HD * HD; e += NTHREADS) p.h_out[hoff + e] = p.h_in ? p.h_in[hoff + e] : 0.f;
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tm, TMEM_COLS);
}

template <typename Tin, bool MUL>
int launch_chunk_t(const ChunkArgs& a, int nblocks, cudaStream_t stream) {
  auto k = dplr_chunk_kernel<Tin, MUL>;
  WKVM_CUDA_TRY(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
  k<<<nblocks, NTHREADS, SMEM_BYTES, stream>>>(a);
  return cudaGetLastError() == cudaSuccess ? WKVM_OK : WKVM_ERR_CUDA;
}

template <bool MUL>
int launch_chunk(const ChunkArgs& a, int nblocks, int dtype, cudaStream_t stream) {
  switch (dtype) {
    case WKVM_DTYPE_F32: return launch_chunk_t<float, MUL>(a, nblocks, stream);
    case WKVM_DTYPE_BF16: return launch_chunk_t<__nv_bfloat16, MUL>(a, nblocks, stream);
    case WKVM_DTYPE_F16: return launch_chunk_t<__half, MUL>(a, nblocks, stream);
    default: return WKVM_ERR_DTYPE;
  }
}

bool al16(const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; }

}  // namespace
}  // namespace wkvm

extern "C" int wkvm_fused_recurrent_dplr(const void*, const void*, const void*, const void*,
                                         const void*, const void*, void*, const float*, float*,
                                         const int64_t*, int32_t, int32_t, int32_t, int32_t,
                                         int32_t, float, int32_t, int32_t*, wkvm_stream_t);
extern "C" int wkvm_wkv7_decode_slots(const void*, const void*, const void*, const void*,
                                      const void*, const void*, void*, float*, int64_t,
                                      const int32_t*, int32_t, int32_t, int32_t, int32_t,
                                      int32_t, int32_t, int32_t*, wkvm_stream_t);

extern "C" int wkvm_chunk_dplr(const void* r, const void* w, const void* k, const void* v,
                               const void* a, const void* b, void* o, const float* h0,
                               float* ht, const int64_t* cu_seqlens, int32_t B, int32_t T,
                               int32_t H, int32_t K, int32_t V, float scale, int32_t dtype,
                               int32_t* status, wkvm_stream_t stream) {
  if (K != 64 || V != 64)  // other head sizes run the recurrent kernel
    return wkvm_fused_recurrent_dplr(r, w, k, v, a, b, o, h0, ht, cu_seqlens, B, T, H, K, V,
                                     scale, dtype, status, stream);
  if (B < 0 || T < 0 || H <= 0) return WKVM_ERR_INVALID_ARG;
  if (B == 0) return WKVM_OK;
  if (!r || !w || !k || !v || !a || !b || !o) return WKVM_ERR_INVALID_ARG;
  if ((h0 && !wkvm::al16(h0)) || (ht && !wkvm::al16(ht)) || !wkvm::al16(o)) return WKVM_ERR_ALIGN;
  wkvm::ChunkArgs args{r, w, k, v, a, b, o, h0, ht, nullptr, 0, cu_seqlens, T, H, scale, status};
  return wkvm::launch_chunk<false>(args, B * H, dtype, (cudaStream_t)stream);
}

extern "C" int wkvm_wkv7_prefill_slots(const void* r, const void* w, const void* k, const void* v,
                                       const void* kk, const void* a, void* o, float* bank_layer,
                                       int64_t num_slots, const int32_t* slot_ids,
                                       const int64_t* cu_seqlens, int32_t B, int32_t T, int32_t H,
                                       int32_t K, int32_t V, int32_t dtype, int32_t* status,
                                       wkvm_stream_t stream) {
  if (!bank_layer || num_slots <= 0 || (B > 0 && !slot_ids)) return WKVM_ERR_INVALID_ARG;
  if (K != 64 || V != 64) {
    if (cu_seqlens) return WKVM_ERR_SHAPE;
    return wkvm_wkv7_decode_slots(r, w, k, v, kk, a, o, bank_layer, num_slots, slot_ids, B, T,
                                  H, K, V, dtype, status, stream);
  }
  if (B < 0 || T < 0 || H <= 0) return WKVM_ERR_INVALID_ARG;
  if (B == 0) return WKVM_OK;
  if (!r || !w || !k || !v || !kk || !a || !o) return WKVM_ERR_INVALID_ARG;
  if (!wkvm::al16(bank_layer) || !wkvm::al16(o)) return WKVM_ERR_ALIGN;
  wkvm::ChunkArgs args{r, w, k, v, kk, a, o, bank_layer, bank_layer, slot_ids, num_slots,
                       cu_seqlens, T, H, 1.0f, status};
  return wkvm::launch_chunk<true>(args, B * H, dtype, (cudaStream_t)stream);
}
