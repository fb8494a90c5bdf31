// Chunked (WY / UT-transform) prefill of the RWKV-7 DPLR recurrence on the
// sm_100a tensor core (tcgen05.mma kind::tf32, fp32 accumulators in TMEM).
//
// One CTA owns one (sequence, head) and walks its 64-token chunks in order,
// keeping every intermediate on chip; HBM sees only the 16-bit inputs, the
// 16-bit outputs and the fp32 state once in and once out.
//
// Per chunk (rows t, s = tokens, k, j = key index, v = value index; G = the
// inclusive cumulative log-decay, Gx = G - w the exclusive one, g0 = G at the
// chunk midpoint as a scaling reference, C = the last row):
//   [a e^(Gx-g0); r e^(G-g0)] x [k e^(g0-G); b e^(g0-G)]^T
//        -> A_ak (s<t), A_ab (s<t), A_qk (s<=t), A_qb (s<=t)         (MMA 1)
//   V^T x A_ak^T = (A_ak V)^T                                         (MMA 2)
//   T = (I - A_ab)^-1, blocked 16 -> 32 -> 64 inverse on the CUDA cores
//   [(A_ak V)^T; (a e^Gx)^T] x T^T = [U~^T; W^T]                      (MMA S)
//   [Bh^T; A_qb] x W                                                  (MMA 3a)
//   [Bh^T; A_qb] x U~ + [Kh^T; A_qk] x V = [N; O_intra]               (MMA 3b)
//        with Kh = k e^(G_C - G), Bh = b e^(G_C - G)
//   M = diag(e^G_C) + Bh^T W,  P = r e^G + A_qb W
//   [S'; O] = [M; P] x S + [N; O_intra]                               (MMA 4)
//
// A operands live in tensor memory where they are produced there: MMA 1's
// accumulator is masked in place and its lower half feeds MMA 3; MMA 2's
// result, completed by (a e^Gx)^T, feeds MMA S; MMA 3's accumulator becomes
// MMA 4's A operand. TMEM: [0,64) a~/r~ -> [(A_ak V)^T; (a e^Gx)^T] ->
// [M; P]; [64,192) MMA 1's result, later [Kh^T | Bh^T] in its upper lanes;
// [192,256) [U~^T; W^T] -> [N; O_intra] -> [S'; O]; [256,320) r e^G.
//
// Algebra and operand orientation are this file's own; the chunk recurrence
// is the one fla's chunk_dplr_delta_rule implements
// (fla/ops/generalized_delta_rule/dplr/chunk.py:33-135, reference
// dplr_chunkwise in .../dplr/naive.py:41-101). tf32 operands keep the result
// within 2e-3 of the fp32 recurrence after 4096 tokens; bf16 operands do not.
#include "chunk_common.cuh"
#include "tma.cuh"

namespace wkvm {
namespace {

constexpr int CH = 64;             // chunk length
constexpr int HD = 64;             // head dim (K == V)
constexpr int NTHREADS = 512;      // four warps per TMEM lane quarter
constexpr int CW = 64 / (NTHREADS / 128);  // columns of a row each thread takes
constexpr int NIN = 6;             // r, w, k, v, x5, x6 input streams
constexpr uint32_t LBO = 128;      // K-adjacent core matrices
constexpr uint32_t SBO = 2048;     // 8-row groups of a 64-wide K tile
constexpr uint32_t LBO_S = 144;    // S^T: padded so column writes hit distinct banks
constexpr uint32_t SBO_S = 16 * LBO_S;
constexpr uint32_t KSTEP = 2 * LBO;  // 8 tf32 (32 bytes) of K per MMA
constexpr int RS = 68;             // row stride (floats) of row-major scratch
constexpr uint32_t STG_TILE = CH * 128;  // one input stream's chunk: 64 rows x 128 B (TMA box)

// shared-memory regions (bytes)
constexpr uint32_t S_STG = 0;                                   // raw inputs [6][64 rows], swizzled
constexpr uint32_t S_G = S_STG + NIN * STG_TILE;                // G row-major (stride RS)
constexpr uint32_t S_AK = S_G + CH * RS * 4;                    // A_ak tile (row t, K = s)
constexpr uint32_t S_AAB = S_AK + CH * RS * 4;                  // A_ab row-major
constexpr uint32_t S_TT = S_AAB + CH * RS * 4;                  // (I - A_ab)^-1 tile (row t', K = t)
constexpr uint32_t S_RB = S_TT + CH * RS * 4;                   // [k~; b~] -> [W^T; U~^T]
constexpr uint32_t S_VT = S_RB + 2 * 8 * SBO;                   // V^T
constexpr uint32_t S_ST = S_VT + 8 * SBO;                       // S^T (the running state)
constexpr uint32_t S_TR = S_ST + 8 * SBO_S;                     // scratch of the inverse
constexpr uint32_t SMEM_USED = S_TR + CH * RS * 4;
constexpr uint32_t SMEM_BYTES = SMEM_USED + 1024;               // + alignment slack
static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");

// The shared-memory footprint allows one CTA per SM, so the CTA takes all
// 512 TMEM columns.
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t T_A1 = 0;     // a~/r~, then A_ak V, then [M; P]
constexpr uint32_t T_D1 = 64;    // MMA 1 accumulator (128 columns)
constexpr uint32_t T_D3 = 192;   // [N; O_intra] -> [S'; O]
constexpr uint32_t T_RG = 256;   // r e^G, rows in lanes 64..127

enum { IN_R = 0, IN_W, IN_K, IN_V, IN_5, IN_6 };

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

__device__ __forceinline__ void kst4(uint8_t* tile, int row, int k, float4 x) {
  *reinterpret_cast<float4*>(tile + tc::kmajor_off(row, k, LBO, SBO)) = x;
}
__device__ __forceinline__ void st4(float* p, const float* x) {
  *reinterpret_cast<float4*>(p) = make_float4(x[0], x[1], x[2], x[3]);
}

// The six input streams of a chunk, one TMA box each (64 tokens x 64 x 16 bit).
struct InMaps {
  CUtensorMap m[NIN];
};

// Element k of row t of staged input stream `in` (128-byte swizzled tile).
template <typename T>
__device__ __forceinline__ float stg(const uint8_t* sm, int in, int t, int k) {
  return to_f32(*reinterpret_cast<const T*>(sm + S_STG + in * STG_TILE +
                                            tma::sw128_off(t, (uint32_t)k * 2)));
}

// 8 consecutive 16-bit inputs of row t starting at column k (k % 8 == 0).
template <typename T>
__device__ __forceinline__ void stg8(const uint8_t* sm, int in, int t, int k, float (&x)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(sm + S_STG + in * STG_TILE +
                                                  tma::sw128_off(t, (uint32_t)k * 2));
  const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
  for (int i = 0; i < 8; ++i) x[i] = to_f32(e[i]);
}

template <typename T>
__device__ __forceinline__ void store_row(T* dst, const float (&v)[CW]) {
#pragma unroll
  for (int i = 0; i < CW; i += 8) {
    uint4 u;
    T* e = reinterpret_cast<T*>(&u);
#pragma unroll
    for (int j = 0; j < 8; ++j) e[j] = from_f32<T>(v[i + j]);
    *reinterpret_cast<uint4*>(dst + i) = u;
  }
}

__device__ __forceinline__ void sync_tc() {
  tc::fence_smem_to_async();
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
}

// b from the two extra input streams (MUL: kk, a_gate -> b = kk * a_gate in
// fp32 as fla's fused_mul_recurrent_rwkv7 does; otherwise b itself).
template <typename T, bool MUL>
__device__ __forceinline__ float in_b(const uint8_t* sm, int t, int k) {
  const float x6 = stg<T>(sm, IN_6, t, k);
  return MUL ? stg<T>(sm, IN_5, t, k) * x6 : x6;
}

// Thread roles: warp w serves TMEM lane quarter (w & 3); the four warps of a
// quarter split the 64 columns of each row into groups g = w >> 2. A thread's
// accumulator row is l = 32 (w & 3) + lane; rows 0..63 ("lo") carry the
// a/k-side and state rows, rows 64..127 the r/b-side and output rows.
template <typename Tin, bool MUL>
__global__ void __launch_bounds__(NTHREADS, 1)
dplr_chunk_kernel(ChunkArgs p, const __grid_constant__ InMaps maps) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                           ~static_cast<uintptr_t>(1023));
  __shared__ uint64_t mbar;
  __shared__ uint64_t tma_bar;  // input tiles of the next chunk landed
  __shared__ uint32_t tmem_slot;
  __shared__ float s_gc[HD];    // e^{G_C}
  __shared__ float s_ref[HD];   // G at the chunk midpoint
  __shared__ float s_eref[HD];  // e^{G at the midpoint}
  __shared__ float s_seg[NTHREADS / HD][HD];  // per-segment totals of the w scan

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quarter = warp & 3;
  const int g = warp >> 2;                 // column group
  const int l = quarter * 32 + lane;       // accumulator row / TMEM lane
  const bool lo = l < 64;
  const int r64 = l & 63;
  const int c0 = g * CW;                   // first column of this thread's half
  const int H = p.H;
  const int n = blockIdx.x / H;
  const int hh = blockIdx.x - n * H;

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
  Tin* __restrict__ go = static_cast<Tin*>(p.o);
  float* Grow = reinterpret_cast<float*>(sm + S_G);
  float* Aab = reinterpret_cast<float*>(sm + S_AAB);

  if (warp == 0) {
    tc::tmem_alloc(&tmem_slot, TMEM_COLS);
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    tc::mbar_init(&mbar, 1);
    tc::mbar_init(&tma_bar, 1);
    tc::fence_mbar_init();
#pragma unroll
    for (int i = 0; i < NIN; ++i) tma::prefetch_map(&maps.m[i]);
  }
  // S^T[v][k] = h[k][v]; thread k = tid & 63 writes a quarter of column k
  for (int e = tid; e < HD * HD; e += NTHREADS) {
    const int k = e & 63, v = e >> 6;
    const float x = p.h_in ? p.h_in[hoff + k * HD + v] : 0.f;
    *reinterpret_cast<float*>(sm + S_ST + tc::kmajor_off(v, k, LBO_S, SBO_S)) = x;
  }
  sync_tc();
  const uint32_t tm = tmem_slot;
  const uint32_t tq = tc::tmem_addr(tm, quarter * 32, 0);  // this warp's lane quarter
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
  const uint32_t idesc64 = tc::idesc_tf32(128, 64);
  const uint32_t idesc128 = tc::idesc_tf32(128, 128);

  // Lane 0 of the last warp issues the TMA loads of chunk c's six 64 x 64 input tiles (one
  // box per stream, no multicast), counted on tma_bar. Rows past the end of
  // the sequence are zeroed after they land (see the loop head).
  uint32_t tphase = 0;
  bool tma_pending = false;
  auto stage = [&](int c) {
    if (tid == NTHREADS - 32) {  // off warp 0, which issues the MMAs and polls their barrier
      tc::mbar_expect_tx(&tma_bar, NIN * STG_TILE);
      const int tok = (int)(bos + (int64_t)c * CH);
#pragma unroll
      for (int i = 0; i < NIN; ++i)
        tma::load_rows(sm + S_STG + i * STG_TILE, &maps.m[i], hh, tok, &tma_bar);
    }
    tma_pending = true;
  };
  if (nchunks > 0) stage(0);

  for (int c = 0; c < nchunks; ++c) {
    const int64_t tok0 = bos + (int64_t)c * CH;
    const int64_t rem = len - (int64_t)c * CH;
    const int clen = rem < CH ? (int)rem : CH;
    const bool last = (c == nchunks - 1);

    // ---- the chunk's raw inputs were staged by the previous iteration (or
    //      before the loop); wait for the TMA loads to land (warp 0 polls)
    {
      const bool ok = warp != 0 || tc::mbar_wait(&tma_bar, tphase);
      if (__syncthreads_or(!ok)) {  // the loads stay pending: waited for once more below
        if (tid == 0) report(p.status, WKVM_ERR_TIMEOUT);
        failed = true;
        break;
      }
      tphase ^= 1u;
      tma_pending = false;
      if (clen < CH) {  // rows past the sequence end hold the next one's tokens
        for (int e = tid; e < NIN * (CH - clen) * 8; e += NTHREADS) {
          const int in = e / ((CH - clen) * 8), rest = e - in * (CH - clen) * 8;
          *reinterpret_cast<uint4*>(sm + S_STG + in * STG_TILE + (clen + (rest >> 3)) * 128 +
                                    (rest & 7) * 16) = make_uint4(0, 0, 0, 0);
        }
        __syncthreads();
      }
    }

    // ---- E1: inclusive scan of w down each column by all threads: thread
    //      (column k = tid & 63, segment tid >> 6) scans 8 tokens, then adds
    //      the totals of the segments above; V^T is written meanwhile.
    {
      const int k = tid & 63, seg = tid >> 6, t0 = seg * 8;
      float acc = 0.f;
#pragma unroll
      for (int t = t0; t < t0 + 8; ++t) {
        acc += stg<Tin>(sm, IN_W, t, k);
        Grow[t * RS + k] = acc;
      }
      s_seg[seg][k] = acc;
#pragma unroll
      for (int t = t0; t < t0 + 8; t += 4)
        kst4(sm + S_VT, k, t,
             make_float4(stg<Tin>(sm, IN_V, t, k), stg<Tin>(sm, IN_V, t + 1, k),
                         stg<Tin>(sm, IN_V, t + 2, k), stg<Tin>(sm, IN_V, t + 3, k)));
      __syncthreads();
      float off = 0.f;
      for (int j = 0; j < seg; ++j) off += s_seg[j][k];
      if (seg > 0) {
#pragma unroll
        for (int t = t0; t < t0 + 8; ++t) Grow[t * RS + k] += off;
      }
    }
    __syncthreads();
    if (tid < 128) {
      const int k = tid & 63;
      if (tid < 64) {
        const float mid = Grow[31 * RS + k];
        s_ref[k] = mid;
        s_eref[k] = __expf(mid);
      } else {
        const float mid = Grow[31 * RS + k];
        const float gc = Grow[63 * RS + k];
        s_gc[k] = __expf(gc);
        // exp(+-(G - G_mid)) must stay finite in fp32 (e^88); RWKV-7's
        // decay (w >= -0.61 per token) keeps the span under 20.
        if (fmaxf(fabsf(Grow[k] - mid), fabsf(gc - mid)) > 80.f)
          report(p.status, WKVM_ERR_UNSUPPORTED);
      }
    }
    __syncthreads();

    // ---- E2: rows. lo rows t: a~ -> TMEM, k~ -> B tile row t;
    //          hi rows t: r~ -> TMEM, b~ -> B tile row 64+t, r e^G -> TMEM.
    {
      const int t = r64;
      float av[CW], xg[CW];
#pragma unroll
      for (int k8 = 0; k8 < CW; k8 += 8) {
        const int k0 = c0 + k8;
        float x[8], wv[8], y[8], z[8], gt[8];
        stg8<Tin>(sm, IN_W, t, k0, wv);
        stg8<Tin>(sm, IN_5, t, k0, x);
        if (lo) {
          stg8<Tin>(sm, IN_K, t, k0, y);
        } else {
          stg8<Tin>(sm, IN_R, t, k0, y);
          stg8<Tin>(sm, IN_6, t, k0, z);
        }
        *reinterpret_cast<float4*>(&gt[0]) = *reinterpret_cast<const float4*>(&Grow[t * RS + k0]);
        *reinterpret_cast<float4*>(&gt[4]) = *reinterpret_cast<const float4*>(&Grow[t * RS + k0 + 4]);
        float bt[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int k = k0 + i;
          const float ref = s_ref[k];
          const float er = s_eref[k];
          if (lo) {
            const float a = MUL ? -x[i] : x[i];
            const float ea = a * __expf(gt[i] - wv[i] - ref);  // a e^{Gx - g0}
            const float einv = __expf(ref - gt[i]);            // e^{g0 - G}
            av[k8 + i] = ea;
            xg[k8 + i] = 0.f;
            bt[i] = y[i] * einv;                        // k~
          } else {
            const float e = __expf(gt[i] - ref);       // e^{G - g0}
            const float einv = __fdividef(1.f, e);     // e^{g0 - G}
            const float rr = y[i] * p.scale * e;       // r~
            av[k8 + i] = rr;
            xg[k8 + i] = rr * er;                       // r e^G
            const float b = MUL ? x[i] * z[i] : z[i];
            bt[i] = b * einv;                           // b~
          }
        }
        kst4(sm + S_RB, l, k0, make_float4(bt[0], bt[1], bt[2], bt[3]));
        kst4(sm + S_RB, l, k0 + 4, make_float4(bt[4], bt[5], bt[6], bt[7]));
      }
      tc::tmem_st(tq + T_A1 + c0, av);
      if (!lo) tc::tmem_st(tq + T_RG + c0, xg);
      tc::tmem_st_wait();
    }
    sync_tc();

    // ---- MMA 1: [a~; r~](TMEM) x [k~; b~]^T -> D1
    if (tid == 0) {
      const uint64_t b0 = tc::smem_desc(tc::smem_u32(sm + S_RB), LBO, SBO);
#pragma unroll
      for (int kk = 0; kk < HD / 8; ++kk)
        tc::mma_tf32_ta(tm + T_D1, tm + T_A1 + kk * 8, tc::desc_add(b0, kk * KSTEP), idesc128,
                        kk > 0);
      tc::mma_commit(&mbar);
    }
    if (!wait_mma()) { failed = true; break; }

    // ---- mask in place: rows t of the top half keep s < t, bottom s <= t.
    //      A_ak (top, left) -> shared-memory tile (row t, K = s) for MMA 2;
    //      A_ab (top, right) -> row-major shared memory for the inverse;
    //      A_qk, A_qb (bottom) stay in TMEM as A operands of MMA 3.
    {
      const int t = r64;
#pragma unroll 1
      for (int h2 = 0; h2 < 2; ++h2) {  // h2 = 0: x k~ columns, 1: x b~ columns
        float x[CW];
        const uint32_t ta = tq + T_D1 + h2 * 64 + c0;
        tc::tmem_ld(ta, x);
#pragma unroll
        for (int i = 0; i < CW; ++i) {
          const int s = c0 + i;
          const bool keep = lo ? (s < t) : (s <= t);
          x[i] = keep ? x[i] : 0.f;
        }
        if (lo && h2 == 1) {
#pragma unroll
          for (int i = 0; i < CW; i += 4) st4(&Aab[t * RS + c0 + i], &x[i]);
        } else if (lo) {
#pragma unroll
          for (int i = 0; i < CW; i += 4)
            kst4(sm + S_AK, t, c0 + i, make_float4(x[i], x[i + 1], x[i + 2], x[i + 3]));
        } else {
          tc::tmem_st(ta, x);
        }
      }
      tc::tmem_st_wait();
    }
    sync_tc();

    // ---- MMA 2: V^T x A_ak^T -> T_A1 lanes v = (A_ak V)^T. The A operand's
    //      rows 64..127 run into the next tile (S^T) and give unused rows.
    if (tid == 0) {
      const uint64_t a0 = tc::smem_desc(tc::smem_u32(sm + S_VT), LBO, SBO);
      const uint64_t b0 = tc::smem_desc(tc::smem_u32(sm + S_AK), LBO, SBO);
#pragma unroll
      for (int kk = 0; kk < CH / 8; ++kk)
        tc::mma_tf32(tm + T_A1, tc::desc_add(a0, kk * KSTEP), tc::desc_add(b0, kk * KSTEP),
                     idesc64, kk > 0);
      tc::mma_commit(&mbar);
    }

    // ---- threads 256..511: T = (I - A_ab)^-1 as a K-major tile (row t',
    //      K = t), while MMA 2 runs; threads 0..255, the column phase (thread =
    //      column k, 32 tokens): lo lanes Kh^T, Bh^T -> TMEM lanes k of D1's
    //      halves (A_ak, A_ab spent) at once; hi lanes, once MMA 2 is done,
    //      (a e^Gx)^T -> T_A1 lanes 64+k, under (A_ak V)^T in lanes 0..63.
    //      The inverse is the longer of the two, so it goes to the warps that
    //      did not just issue MMA 2.
    bool ok2 = true;
    if (tid >= 256) {
      chunkc::tri_inverse64(Aab, reinterpret_cast<float*>(sm + S_TR), sm + S_TT, tid - 256, 256);
    } else if (!lo && !(ok2 = tc::mbar_wait(&mbar, phase))) {
      // reported below (only the hi lanes write where MMA 2 writes)
    } else {
      tc::fence_after_sync();
      const int k = r64, cc0 = (warp >> 2) * 32;
      if (lo) {  // two halves of 16 tokens keep the live registers down
        const float gc = Grow[63 * RS + k];
#pragma unroll
        for (int hh = 0; hh < 32; hh += 16) {
          float x[16], y[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int t = cc0 + hh + i;
            const float e = __expf(gc - Grow[t * RS + k]);
            x[i] = stg<Tin>(sm, IN_K, t, k) * e;
            y[i] = in_b<Tin, MUL>(sm, t, k) * e;
          }
          tc::tmem_st16(tq + T_D1 + cc0 + hh, x);
          tc::tmem_st16(tq + T_D1 + 64 + cc0 + hh, y);
        }
      } else {
        float x[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int t = cc0 + i;
          const float a = stg<Tin>(sm, IN_5, t, k);
          x[i] = (MUL ? -a : a) * __expf(Grow[t * RS + k] - stg<Tin>(sm, IN_W, t, k));
        }
        tc::tmem_st32(tq + T_A1 + cc0, x);
      }
      tc::tmem_st_wait();
    }
    phase ^= 1u;
    tc::fence_smem_to_async();
    tc::fence_before_sync();
    if (__syncthreads_or(!ok2)) {
      if (tid == 0) report(p.status, WKVM_ERR_TIMEOUT);
      failed = true;
      break;
    }
    tc::fence_after_sync();

    // ---- MMA S: [(A_ak V)^T; (a e^Gx)^T] x T^T -> T_D3 = [U~^T; W^T]
    if (tid == 0) {
      const uint64_t b0 = tc::smem_desc(tc::smem_u32(sm + S_TT), LBO, SBO);
#pragma unroll
      for (int kk = 0; kk < CH / 8; ++kk)
        tc::mma_tf32_ta(tm + T_D3, tm + T_A1 + kk * 8, tc::desc_add(b0, kk * KSTEP), idesc64,
                        kk > 0);
      tc::mma_commit(&mbar);
    }
    // The staged inputs and G are spent: stage the next chunk now so its
    // copies overlap the rest of this one (after MMA S is issued, so that the
    // issuing thread does not queue behind its share of the copies).
    if (c + 1 < nchunks) stage(c + 1);
    if (!wait_mma()) { failed = true; break; }
    {  // [W^T; U~^T] B tile: lane l < 64 holds U~^T row l, lane 64+j holds W^T row j
      float x[CW];
      tc::tmem_ld(tq + T_D3 + c0, x);
      const int row = lo ? 64 + l : l - 64;
#pragma unroll
      for (int i = 0; i < CW; i += 4)
        kst4(sm + S_RB, row, c0 + i, make_float4(x[i], x[i + 1], x[i + 2], x[i + 3]));
    }
    sync_tc();

    // ---- MMA 3a: [Bh^T; A_qb] x W -> T_A1 ; MMA 3b: [Bh^T; A_qb] x U~
    //      + [Kh^T; A_qk] x V -> T_D3
    if (tid == 0) {
      const uint32_t w0 = tc::smem_u32(sm + S_RB);
      const uint32_t u0 = w0 + 8 * SBO;
      const uint32_t v0 = tc::smem_u32(sm + S_VT);
      const uint64_t wd = tc::smem_desc(w0, LBO, SBO), ud = tc::smem_desc(u0, LBO, SBO);
      const uint64_t vd = tc::smem_desc(v0, LBO, SBO);
#pragma unroll
      for (int kk = 0; kk < CH / 8; ++kk)
        tc::mma_tf32_ta(tm + T_A1, tm + T_D1 + 64 + kk * 8, tc::desc_add(wd, kk * KSTEP), idesc64,
                        kk > 0);
#pragma unroll
      for (int kk = 0; kk < CH / 8; ++kk)
        tc::mma_tf32_ta(tm + T_D3, tm + T_D1 + 64 + kk * 8, tc::desc_add(ud, kk * KSTEP), idesc64,
                        kk > 0);
#pragma unroll
      for (int kk = 0; kk < CH / 8; ++kk)
        tc::mma_tf32_ta(tm + T_D3, tm + T_D1 + kk * 8, tc::desc_add(vd, kk * KSTEP), idesc64,
                        true);
      tc::mma_commit(&mbar);
    }
    if (!wait_mma()) { failed = true; break; }

    // ---- M = diag(e^G_C) + Bh^T W (lanes k), P = r e^G + A_qb W (lanes 64+t)
    {
      float x[CW];
      const uint32_t ta = tq + T_A1 + c0;
      tc::tmem_ld(ta, x);
      if (lo) {
        const int k = r64;
        const float d = s_gc[k];
#pragma unroll
        for (int i = 0; i < CW; ++i) x[i] += (c0 + i == k) ? d : 0.f;
      } else {
        float rg[CW];
        tc::tmem_ld(tq + T_RG + c0, rg);
#pragma unroll
        for (int i = 0; i < CW; ++i) x[i] += rg[i];
      }
      tc::tmem_st(ta, x);
      tc::tmem_st_wait();
    }
    sync_tc();

    // ---- MMA 4: [S'; O] = [M; P] x S + [N; O_intra]
    if (tid == 0) {
      const uint64_t s0 = tc::smem_desc(tc::smem_u32(sm + S_ST), LBO_S, SBO_S);
#pragma unroll
      for (int kk = 0; kk < HD / 8; ++kk)
        tc::mma_tf32_ta(tm + T_D3, tm + T_A1 + kk * 8, tc::desc_add(s0, kk * 2 * LBO_S), idesc64,
                        true);
      tc::mma_commit(&mbar);
    }
    if (!wait_mma()) { failed = true; break; }

    {
      float x[CW];
      tc::tmem_ld(tq + T_D3 + c0, x);
      if (lo) {
        const int k = r64;  // S'[k][v]: column k of S^T
#pragma unroll
        for (int i = 0; i < CW; ++i)
          *reinterpret_cast<float*>(sm + S_ST + tc::kmajor_off(c0 + i, k, LBO_S, SBO_S)) = x[i];
        if (last && p.h_out) {
          float* dst = p.h_out + hoff + k * HD + c0;
#pragma unroll
          for (int i = 0; i < CW; i += 4)
            st_stream_f4(dst + i, make_float4(x[i], x[i + 1], x[i + 2], x[i + 3]));
        }
      } else {
        const int t = r64;
        if (t < clen) store_row(go + ((tok0 + t) * H + hh) * HD + c0, x);
      }
    }
    // the next chunk's first barrier (its TMA wait) orders these TMEM reads
    // and S^T writes before anything that touches them again: T_D3 is next
    // written by MMA S and S^T next read by MMA 4, each behind a fenced
    // barrier of its own
    tc::fence_before_sync();
  }

  // no TMA load may still target this CTA's shared memory
  if (tma_pending && !(warp != 0 || tc::mbar_wait(&tma_bar, tphase)) && tid == 0)
    report(p.status, WKVM_ERR_TIMEOUT);
  __syncthreads();
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

// `tokens`: rows of the activation tensors (B * T, or the varlen total T).
template <typename Tin, bool MUL>
int launch_chunk_t(const ChunkArgs& a, int nblocks, int64_t tokens, cudaStream_t stream) {
  auto k = dplr_chunk_kernel<Tin, MUL>;
  InMaps maps;
  const void* in[NIN] = {a.p0, a.p1, a.p2, a.p3, a.p4, a.p5};
  for (int i = 0; i < NIN; ++i) {
    const int rc = tma::encode_rows(&maps.m[i], in[i], tokens, a.H, HD, CH);
    if (rc != WKVM_OK) return rc;
  }
  WKVM_CUDA_TRY(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
  k<<<nblocks, NTHREADS, SMEM_BYTES, stream>>>(a, maps);
  return cudaGetLastError() == cudaSuccess ? WKVM_OK : WKVM_ERR_CUDA;
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
extern "C" int wkvm_fused_mul_recurrent_rwkv7(const void*, const void*, const void*, const void*,
                                              const void*, const void*, void*, const float*,
                                              float*, const int64_t*, int32_t, int32_t, int32_t,
                                              int32_t, int32_t, float, int32_t, int32_t*,
                                              wkvm_stream_t);

namespace {
// The tensor-core path stages 16-bit rows with 16-byte copies.
bool chunk_path_ok(int K, int V, int dtype, const void* const* ptrs, int n) {
  if (K != 64 || V != 64) return false;
  if (dtype != WKVM_DTYPE_BF16 && dtype != WKVM_DTYPE_F16) return false;
  for (int i = 0; i < n; ++i)
    if (!wkvm::al16(ptrs[i])) return false;
  return true;
}
}  // namespace

extern "C" int wkvm_chunk_dplr(const void* r, const void* w, const void* k, const void* v,
                               const void* a, const void* b, void* o, const float* h0,
                               float* ht, const int64_t* cu_seqlens, int32_t B, int32_t T,
                               int32_t H, int32_t K, int32_t V, float scale, int32_t dtype,
                               int32_t* status, wkvm_stream_t stream) {
  const void* ptrs[7] = {r, w, k, v, a, b, o};
  if (!chunk_path_ok(K, V, dtype, ptrs, 7))  // other shapes/dtypes: recurrent kernel
    return wkvm_fused_recurrent_dplr(r, w, k, v, a, b, o, h0, ht, cu_seqlens, B, T, H, K, V,
                                     scale, dtype, status, stream);
  if (B < 0 || T < 0 || H <= 0) return WKVM_ERR_INVALID_ARG;
  if (B == 0) return WKVM_OK;
  if (!r || !w || !k || !v || !a || !b || !o) return WKVM_ERR_INVALID_ARG;
  const int64_t tokens = cu_seqlens ? (int64_t)T : (int64_t)B * T;
  if (tokens == 0) return wkvm_fused_recurrent_dplr(r, w, k, v, a, b, o, h0, ht, cu_seqlens, B, T,
                                                    H, K, V, scale, dtype, status, stream);
  if ((h0 && !wkvm::al16(h0)) || (ht && !wkvm::al16(ht))) return WKVM_ERR_ALIGN;
  wkvm::ChunkArgs args{r, w, k, v, a, b, o, h0, ht, nullptr, 0, cu_seqlens, T, H, scale, status};
  if (dtype == WKVM_DTYPE_BF16)
    return wkvm::launch_chunk_t<__nv_bfloat16, false>(args, B * H, tokens, (cudaStream_t)stream);
  return wkvm::launch_chunk_t<__half, false>(args, B * H, tokens, (cudaStream_t)stream);
}

extern "C" int wkvm_wkv7_prefill_slots(const void* r, const void* w, const void* k, const void* v,
                                       const void* kk, const void* a, void* o, float* bank_layer,
                                       int64_t num_slots, const int32_t* slot_ids,
                                       const int64_t* cu_seqlens, int32_t B, int32_t T, int32_t H,
                                       int32_t K, int32_t V, int32_t dtype, int32_t* status,
                                       wkvm_stream_t stream) {
  if (!bank_layer || num_slots <= 0 || (B > 0 && !slot_ids)) return WKVM_ERR_INVALID_ARG;
  const void* ptrs[7] = {r, w, k, v, kk, a, o};
  if (!chunk_path_ok(K, V, dtype, ptrs, 7)) {
    if (cu_seqlens) return WKVM_ERR_UNSUPPORTED;
    return wkvm_wkv7_decode_slots(r, w, k, v, kk, a, o, bank_layer, num_slots, slot_ids, B, T,
                                  H, K, V, dtype, status, stream);
  }
  if (B < 0 || T < 0 || H <= 0) return WKVM_ERR_INVALID_ARG;
  if (B == 0) return WKVM_OK;
  if (!wkvm::al16(bank_layer)) return WKVM_ERR_ALIGN;
  const int64_t tokens = cu_seqlens ? (int64_t)T : (int64_t)B * T;
  if (tokens == 0) return WKVM_OK;  // the slots keep their state
  wkvm::ChunkArgs args{r, w, k, v, kk, a, o, bank_layer, bank_layer, slot_ids, num_slots,
                       cu_seqlens, T, H, 1.0f, status};
  if (dtype == WKVM_DTYPE_BF16)
    return wkvm::launch_chunk_t<__nv_bfloat16, true>(args, B * H, tokens, (cudaStream_t)stream);
  return wkvm::launch_chunk_t<__half, true>(args, B * H, tokens, (cudaStream_t)stream);
}

extern "C" int wkvm_dplr_prefill_slots(const void* r, const void* w, const void* k, const void* v,
                                       const void* a, const void* b, void* o, float* bank_layer,
                                       int64_t num_slots, const int32_t* slot_ids,
                                       const int64_t* cu_seqlens, int32_t B, int32_t T, int32_t H,
                                       int32_t K, int32_t V, float scale, int32_t dtype,
                                       int32_t* status, wkvm_stream_t stream) {
  if (!bank_layer || num_slots <= 0 || (B > 0 && !slot_ids)) return WKVM_ERR_INVALID_ARG;
  const void* ptrs[7] = {r, w, k, v, a, b, o};
  if (!chunk_path_ok(K, V, dtype, ptrs, 7)) return WKVM_ERR_UNSUPPORTED;
  if (B < 0 || T < 0 || H <= 0) return WKVM_ERR_INVALID_ARG;
  if (B == 0) return WKVM_OK;
  if (!wkvm::al16(bank_layer)) return WKVM_ERR_ALIGN;
  const int64_t tokens = cu_seqlens ? (int64_t)T : (int64_t)B * T;
  if (tokens == 0) return WKVM_OK;  // the slots keep their state
  wkvm::ChunkArgs args{r, w, k, v, a, b, o, bank_layer, bank_layer, slot_ids, num_slots,
                       cu_seqlens, T, H, scale, status};
  if (dtype == WKVM_DTYPE_BF16)
    return wkvm::launch_chunk_t<__nv_bfloat16, false>(args, B * H, tokens, (cudaStream_t)stream);
  return wkvm::launch_chunk_t<__half, false>(args, B * H, tokens, (cudaStream_t)stream);
}
