// Two-phase chunked prefill of the gated delta rule (K = V = 128) on the
// sm_100a tensor core (tcgen05.mma kind::tf32, fp32 accumulators in TMEM).
//
// Only a small part of a chunk's work depends on the incoming state, so it is
// split in two launches:
//
//  phase 1, gdn_wy_kernel: one CTA per (chunk, sequence, value head), all
//    chunks at once. Builds the chunk's WY factors and writes one record:
//      A[t][s] = beta_t e^(G_t-G_s) k^_t.k^_s (s < t),  T = (I + A)^-1
//      U = T (beta v),  W = T (beta e^G k^)                     (u = U - W S)
//      Q~ = scale e^G q^,  K~ = e^(G_C-G) k^,
//      A_qk[t][s] = scale e^(G_t-G_s) q^_t.k^_s (s <= t)
//  phase 2, gdn_state_kernel: two CTAs per (sequence, value head), one per
//    half of the value columns, walk the chunks in order with their half of
//    the state S^T (64 rows v, columns k) resident in TMEM (M = 64 tiles):
//      [(W S)^T | (Q~ S)^T] = S^T [W; Q~]^T                    (MMA A)
//      u^T = U^T - (W S)^T,  S^T <- e^(G_C) S^T
//      S^T += u^T K~,  (Q~ S)^T += u^T A_qk^T = O^T            (MMA B)
//
// The derivation (decay first, then the delta update, per token) follows
// fla's recurrence fla/ops/gated_delta_rule/fused_recurrent.py:128-151 and
// the chunk form of fla/ops/gated_delta_rule/chunk.py:29-116; operand
// orientation, record layout and the TMEM-resident state are this file's own.
//
// Records live in a caller-provided workspace; when it is smaller than the
// whole prefill needs, the sequences are processed in windows of chunks and
// the state is carried between windows in the workspace.
#include <type_traits>

#include "chunk_common.cuh"
#include "tma.cuh"

namespace wkvm {

namespace gdnwy {

constexpr int CH = 64, KD = 128, VD = 128;
constexpr uint32_t LBO = 128;
constexpr uint32_t SBO64 = 2048;                 // fp32 tile, K = 64
constexpr uint32_t KSTEP = 2 * LBO;              // 8 tf32 of K per MMA

// record layout (bytes). Every matrix is fp16: the state pass multiplies
// with kind::f16, whose 10-bit significand is the tf32 one; the values are
// unit-scale (normalised q, k; decays <= 1; U = T (beta v)). The operand
// tiles are K-major, no swizzle, 8-row x 16-byte core matrices, LBO 128.
constexpr uint32_t SBOH64 = 1024, SBOH128 = 2048;  // fp16 tiles, K = 64 / K = 128
constexpr uint32_t KSTEP16 = 2 * LBO;              // 16 fp16 of K per MMA
constexpr uint32_t R_WQ = 0;                 // [W; Q~]: 128 rows x K = 128 (k)
constexpr uint32_t R_KT = R_WQ + 32768;      // K~^T: 128 rows (k) x K = 64 (t)
constexpr uint32_t R_AQK = R_KT + 16384;     // A_qk: 64 rows (t) x K = 64 (s)
constexpr uint32_t R_U = R_AQK + 8192;       // U: two v-halves, each 64 rows (t) x 64 v
constexpr uint32_t R_META = R_U + 16384;     // e^(G_C), fp32
constexpr uint32_t REC_BYTES = R_META + 128;
constexpr uint32_t PART_A = R_KT - R_WQ;             // [W; Q~]: MMA A
constexpr uint32_t PART_B = R_U - R_KT;              // K~^T and A_qk: MMA B
constexpr uint32_t PART_U = 64 * 64 * 2;            // one v-half of U: the u pass

// Byte offset of element (row, k) in an fp16 K-major tile.
__host__ __device__ constexpr uint32_t hoff16(int row, int k, uint32_t sbo) {
  return (uint32_t)(row >> 3) * sbo + (uint32_t)(k >> 3) * LBO + (uint32_t)(row & 7) * 16 +
         (uint32_t)(k & 7) * 2;
}

// Eight floats as fp16, one 16-byte store; `mx` keeps the largest magnitude
// written (a record value beyond fp16's range is reported, not stored silently
// as infinity).
__device__ __forceinline__ void st_h8(uint8_t* p, const float* x, float& mx) {
  uint4 u;
  __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    h[i] = __floats2half2_rn(x[2 * i], x[2 * i + 1]);
    mx = fmaxf(mx, fmaxf(fabsf(x[2 * i]), fabsf(x[2 * i + 1])));
  }
  *reinterpret_cast<uint4*>(p) = u;
}
constexpr float kHalfMax = 65504.f;
static_assert(REC_BYTES % 128 == 0 && PART_B % 16 == 0 && PART_U % 16 == 0,
              "record alignment");

}  // namespace gdnwy

namespace {

using namespace gdnwy;
using chunkc::RS;

struct WyArgs {
  const void *q, *k, *v, *g, *beta;
  uint8_t* ws;        // records [nseq][W][HV]
  const int64_t* cu;
  int T, H, HV, w0, W, nseq;
  float scale;
  bool l2norm;
  int* status;
  bool gates_f32;  // g and beta are fp32 (WKVM_GATES_F32)
};

struct StateArgs {
  const uint8_t* ws;
  void* o;
  const float* h_src;   // state entering the window (nullptr: zeros)
  float* h_dst;         // state leaving the window (nullptr: dropped)
  bool src_slots, dst_slots;  // index h_src / h_dst by slot id (else by sequence)
  const int32_t* ids;
  int64_t num_slots;
  const int64_t* cu;
  int T, HV, w0, W;
  int* status;
};

__device__ __forceinline__ void sync_tc() {
  tc::fence_smem_to_async();
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
}

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) &
                                    ~static_cast<uintptr_t>(1023));
}

// ---------------------------------------------------------------- phase 1

constexpr int WY_THREADS = 256;
// Persistent: each CTA works through jobs (chunk, sequence, value head) with a
// two-stage pipeline; job j+1's inputs land while job j computes.
// A stage holds one job's rows as TMA wrote them (six boxes of 64 tokens x
// 64 elements, 128-byte swizzle): the [k; q] tile in two column blocks of
// 128 rows x 128 bytes (block b: columns 64b..64b+63; rows 0..63 k, 64..127
// q) -- directly the K-major operands of the Gram MMA -- then v in two
// column blocks of 64 rows. Once the stage's k and v have been read, its
// first bytes hold -A (row-major), the inverse's scratch and the T tile.
constexpr uint32_t BOX = CH * 128;                    // one TMA box, 8 KiB
constexpr uint32_t ST_QK = 0;                         // 2 blocks x 16 KiB
constexpr uint32_t ST_V = ST_QK + 4 * BOX;            // 2 blocks x 8 KiB
constexpr uint32_t STAGE = ST_V + 2 * BOX;            // 48 KiB
constexpr uint32_t WS_AAB = 0;                        // within the job's stage
constexpr uint32_t WS_TR = WS_AAB + CH * RS * 4;
constexpr uint32_t WS_TT = WS_AAB;                    // written after -A is spent
static_assert(WS_TR + CH * RS * 4 <= STAGE, "inverse scratch outside the stage");
constexpr uint32_t WY_SMEM = 2 * STAGE + 1024;
constexpr int W_ROW = KD + 4;  // row stride (floats) of W staged row-major in a spent stage
static_assert(CH * W_ROW * 4 <= STAGE, "W staging outside the stage");
// TMEM: MMA 1 accumulator, later U^T | (beta v)^T | (beta e^G k^)^T | W^T
constexpr uint32_t WY_TMEM_COLS = 256;
constexpr uint32_t T_D1 = 0, T_AV = 64, T_AK = 128, T_DW = 192;

// Byte offsets within a stage of element (row, col) of the [k; q] tile
// (rows 0..127) and of the v rows (0..63); col % 8 == 0 for 16-byte reads.
__device__ __forceinline__ uint32_t qk_off(int row, int col) {
  return ST_QK + (uint32_t)(col >> 6) * 2 * BOX + tma::sw128_off(row, (uint32_t)(col & 63) * 2);
}
__device__ __forceinline__ uint32_t v_off(int row, int col) {
  return ST_V + (uint32_t)(col >> 6) * BOX + tma::sw128_off(row, (uint32_t)(col & 63) * 2);
}

// TMA descriptions of q, k ([tokens, H, 128]) and v ([tokens, HV, 128]).
struct WyMaps {
  CUtensorMap q, k, v;
};

struct Job {
  int n, hv, cw;   // sequence, value head, chunk within the window
  int64_t tok0;
  int clen;        // tokens in the chunk (0: past the sequence end)
};

__device__ __forceinline__ Job job_of(const WyArgs& p, int j) {
  Job J;
  J.hv = j % p.HV;
  const int r = j / p.HV;
  J.n = r % p.nseq;
  J.cw = r / p.nseq;
  int64_t bos, len;
  if (p.cu) {
    bos = p.cu[J.n];
    len = p.cu[J.n + 1] - bos;
  } else {
    bos = (int64_t)J.n * p.T;
    len = p.T;
  }
  const int64_t rem = len - (int64_t)(p.w0 + J.cw) * CH;
  J.clen = rem <= 0 ? 0 : (rem < CH ? (int)rem : CH);
  J.tok0 = bos + (int64_t)(p.w0 + J.cw) * CH;
  return J;
}

template <typename Tin>
__global__ void __launch_bounds__(WY_THREADS, 2)
gdn_wy_kernel(WyArgs p, int njobs, const __grid_constant__ WyMaps maps) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024(smem_raw);
  __shared__ uint64_t mbar;
  __shared__ uint64_t in_bar[2];  // a stage's TMA loads landed
  __shared__ uint32_t tmem_slot;
  __shared__ float s_beta[CH], s_G[CH], s_eG[CH], s_eGC[CH], s_rk[CH], s_rq[CH];

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quarter = warp & 3, gh = warp >> 2;
  const int l = quarter * 32 + lane;  // TMEM lane
  const bool lo = l < 64;
  const int r64 = l & 63;
  const int H = p.H, HV = p.HV;
  constexpr bool kBf16 = std::is_same<Tin, __nv_bfloat16>::value;

  if (warp == 0) {
    tc::tmem_alloc(&tmem_slot, WY_TMEM_COLS);
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    tc::mbar_init(&mbar, 1);
    tc::mbar_init(&in_bar[0], 1);
    tc::mbar_init(&in_bar[1], 1);
    tc::fence_mbar_init();
    tma::prefetch_map(&maps.q);
    tma::prefetch_map(&maps.k);
    tma::prefetch_map(&maps.v);
  }

  // TMA loads of job J's k, q, v rows into stage st (one thread of the last
  // warp, off warp 0's barrier polls; nothing for a
  // job past its sequence's end). Rows past clen are zeroed once they land.
  uint32_t in_phase = 0u, in_pending = 0u;  // bit st: stage st's parity / a load in flight
  auto stage_in = [&](const Job& J, int st) {
    if (J.clen <= 0) return;
    in_pending |= 1u << st;
    if (tid != WY_THREADS - 32) return;  // lane 0 of the last warp: warp 0 polls barriers
    uint8_t* base = sm + st * STAGE;
    const int hq = J.hv / (HV / H);
    const int tok = (int)J.tok0;
    tc::mbar_expect_tx(&in_bar[st], 6 * BOX);
#pragma unroll
    for (int b = 0; b < 2; ++b) {
      tma::load_rows(base + ST_QK + b * 2 * BOX, &maps.k, hq, tok, &in_bar[st], 64 * b);
      tma::load_rows(base + ST_QK + b * 2 * BOX + BOX, &maps.q, hq, tok, &in_bar[st], 64 * b);
      tma::load_rows(base + ST_V + b * BOX, &maps.v, J.hv, tok, &in_bar[st], 64 * b);
    }
  };
  // per-token decay and beta of job J into warp 0's registers, as raw bits:
  // the conversion to fp32 waits for the load, so it happens at the use
  const bool gf32 = p.gates_f32;
  auto scalars_in = [&](const Job& J, uint32_t (&x)[4]) {
    x[0] = x[1] = x[2] = x[3] = 0u;
    if (warp == 0) {
      const int64_t i0 = (J.tok0 + lane) * HV + J.hv, i1 = (J.tok0 + lane + 32) * HV + J.hv;
      auto raw = [&](const void* b, int64_t i) -> uint32_t {
        return gf32 ? static_cast<const uint32_t*>(b)[i]
                    : (uint32_t) static_cast<const uint16_t*>(b)[i];
      };
      if (lane < J.clen) {
        x[0] = raw(p.g, i0);
        x[2] = raw(p.beta, i0);
      }
      if (lane + 32 < J.clen) {
        x[1] = raw(p.g, i1);
        x[3] = raw(p.beta, i1);
      }
    }
  };
  auto gate = [&](uint32_t bits) -> float {
    if (gf32) return __uint_as_float(bits);
    const uint16_t h = (uint16_t)bits;
    return to_f32(*reinterpret_cast<const Tin*>(&h));
  };

  int j = blockIdx.x;
  Job cur = job_of(p, j < njobs ? j : 0);
  if (j >= njobs) cur.clen = 0;
  uint32_t sc_cur[4], sc_next[4];
  tc::fence_before_sync();
  __syncthreads();  // barriers initialised before the first load
  tc::fence_after_sync();
  stage_in(cur, 0);
  scalars_in(cur, sc_cur);
  const uint32_t tm = tmem_slot;
  const uint32_t tq = tc::tmem_addr(tm, quarter * 32, 0);
  const uint32_t id_gram = tc::idesc_f16(128, 64, kBf16);
  const uint32_t id_s = tc::idesc_tf32(128, 64);

  float rmax = 0.f;  // largest magnitude this thread wrote to an fp16 record
#pragma unroll 1
  for (int it = 0; j < njobs; ++it, j += gridDim.x) {
    const int st = it & 1;
    uint8_t* sg = sm + st * STAGE;
    // prefetch the next job into the other stage (its previous job is done)
    const int jn = j + gridDim.x;
    Job nxt = job_of(p, jn < njobs ? jn : 0);
    if (jn >= njobs) nxt.clen = 0;
    stage_in(nxt, st ^ 1);
    scalars_in(nxt, sc_next);
    const Job J = cur;
    if (J.clen > 0) {
      uint8_t* rec = p.ws + (((int64_t)J.n * p.W + J.cw) * HV + J.hv) * (int64_t)REC_BYTES;
      {  // this job's stage landed (warp 0 polls); rows past clen -> zero
        const bool ok = warp != 0 || tc::mbar_wait(&in_bar[st], (in_phase >> st) & 1u);
        if (__syncthreads_or(!ok)) {  // still pending: waited for once more below
          if (tid == 0) report(p.status, WKVM_ERR_TIMEOUT);
          break;
        }
        in_phase ^= 1u << st;
        in_pending &= ~(1u << st);
        if (J.clen < CH) {
          const int nz = CH - J.clen;  // rows per box to clear, 8 x 16 bytes each
          for (int e = tid; e < 6 * nz * 8; e += WY_THREADS) {
            const int box = e / (nz * 8), rest = e - box * nz * 8;
            const int row = J.clen + (rest >> 3);
            const uint32_t off = box < 4 ? ST_QK + (box >> 1) * 2 * BOX + (box & 1) * BOX
                                         : ST_V + (box - 4) * BOX;
            *reinterpret_cast<uint4*>(sg + off + row * 128 + (rest & 7) * 16) =
                make_uint4(0, 0, 0, 0);
          }
        }
      }
      if (warp == 0) {  // inclusive decay scan
        float a = gate(sc_cur[0]), b = gate(sc_cur[1]);
        s_beta[lane] = gate(sc_cur[2]);
        s_beta[lane + 32] = gate(sc_cur[3]);
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
        const float gc = __shfl_sync(0xffffffffu, b, 31);
        s_G[lane] = a;
        s_G[lane + 32] = b;
        s_eG[lane] = __expf(a);
        s_eG[lane + 32] = __expf(b);
        s_eGC[lane] = __expf(gc - a);
        s_eGC[lane + 32] = __expf(gc - b);
      }
      sync_tc();

      // ---- MMA 1: [k; q] x k^T -> D1 (16-bit operands: the products of
      //      16-bit inputs are exact in the fp32 accumulator)
      if (tid == 0) {
        const uint64_t x0 = tc::smem_desc_sw128(tc::smem_u32(sg + ST_QK));
#pragma unroll
        for (int kk = 0; kk < KD / 16; ++kk) {  // 16 elements (32 bytes) of K per MMA
          const uint64_t x = tc::desc_add(x0, (kk >> 2) * 2 * BOX + (kk & 3) * 32);
          tc::mma_f16(tm + T_D1, x, x, id_gram, kk > 0);
        }
        tc::mma_commit(&mbar);
      }
      {  // squared norms per row (thread: half a row)
        const int r = tid >> 1, half = tid & 1;
        float ss = 0.f;
#pragma unroll
        for (int pc = 0; pc < 8; ++pc) {
          const uint4 u = *reinterpret_cast<const uint4*>(sg + qk_off(r, half * 64 + pc * 8));
          const Tin* e = reinterpret_cast<const Tin*>(&u);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float x = to_f32(e[i]);
            ss = fmaf(x, x, ss);
          }
        }
        ss += __shfl_xor_sync(0xffffffffu, ss, 1);
        if (half == 0) {
          const float f = p.l2norm ? 1.0f / sqrtf(ss + 1e-6f) : 1.f;
          if (r >= 64) s_rq[r - 64] = f * p.scale;
          else s_rk[r] = f;
        }
      }
      __syncthreads();
      const float GC = s_G[CH - 1];
      {  // A operands of MMA S in TMEM (rows v / k, K = s), K~^T and Q~
        const int s0 = gh * 32;
        float x[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int s = s0 + i;
          x[i] = s_beta[s] * to_f32(*reinterpret_cast<const Tin*>(sg + v_off(s, l)));
        }
        tc::tmem_st32(tq + T_AV + s0, x);
        float y[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int s = s0 + i;
          const float kv =
              to_f32(*reinterpret_cast<const Tin*>(sg + qk_off(s, l))) * s_rk[s];
          x[i] = s_beta[s] * s_eG[s] * kv;
          y[i] = s_eGC[s] * kv;
        }
        tc::tmem_st32(tq + T_AK + s0, x);
#pragma unroll
        for (int i = 0; i < 32; i += 8) st_h8(rec + R_KT + hoff16(l, s0 + i, SBOH64), y + i, rmax);
        // Q~ (rows 64..127 of [W; Q~]): piece e -> row t = 8 g + (e & 7), 8
        // columns from (e >> 3) & 15; eight lanes fill 128 contiguous bytes
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          const int e = tid + WY_THREADS * jj;
          const int t = (e >> 7) * 8 + (e & 7), k8 = ((e >> 3) & 15) * 8;
          const uint4 u = *reinterpret_cast<const uint4*>(sg + qk_off(64 + t, k8));
          const Tin* h = reinterpret_cast<const Tin*>(&u);
          const float f = s_rq[t] * s_eG[t];
          float qv[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) qv[i] = to_f32(h[i]) * f;
          st_h8(rec + R_WQ + hoff16(64 + t, k8, SBOH128), qv, rmax);
        }
        tc::tmem_st_wait();
      }
      bool ok = warp != 0 || tc::mbar_wait(&mbar, 0);  // warp 0 polls
      if (__syncthreads_or(!ok)) {  // give the MMA one more bounded wait before TMEM goes
        if (tid == 0) report(p.status, WKVM_ERR_TIMEOUT);
        tc::mbar_wait(&mbar, 0);
        break;
      }
      tc::fence_after_sync();

      // ---- masks: lo rows -> -A (row-major, over the spent stage) for the
      //      inverse; hi rows -> A_qk
      {
        const int t = r64, s0 = gh * 32;
        float x[32];
        tc::tmem_ld32(tq + T_D1 + s0, x);
        const float Gt = s_G[t];
        if (lo) {
          const float f = -s_beta[t] * s_rk[t];
          float* arow = reinterpret_cast<float*>(sg + WS_AAB) + t * RS + s0;
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int s = s0 + i;
            x[i] = s < t ? f * s_rk[s] * __expf(Gt - s_G[s]) * x[i] : 0.f;
          }
#pragma unroll
          for (int i = 0; i < 32; i += 4)
            *reinterpret_cast<float4*>(arow + i) = make_float4(x[i], x[i + 1], x[i + 2], x[i + 3]);
        } else {
          const float f = s_rq[t];
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int s = s0 + i;
            x[i] = s <= t ? f * s_rk[s] * __expf(Gt - s_G[s]) * x[i] : 0.f;
          }
#pragma unroll
          for (int i = 0; i < 32; i += 8) st_h8(rec + R_AQK + hoff16(t, s0 + i, SBOH64), x + i, rmax);
        }
      }
      __syncthreads();
      chunkc::tri_inverse64(reinterpret_cast<const float*>(sg + WS_AAB),
                            reinterpret_cast<float*>(sg + WS_TR), sg + WS_TT, tid);
      sync_tc();

      // ---- MMA S: (beta v)^T T^T = U^T -> D1 ; (beta e^G k^)^T T^T = W^T -> DW
      if (tid == 0) {
        const uint64_t t0 = tc::smem_desc(tc::smem_u32(sg + WS_TT), LBO, SBO64);
#pragma unroll
        for (int kk = 0; kk < CH / 8; ++kk)
          tc::mma_tf32_ta(tm + T_D1, tm + T_AV + kk * 8, tc::desc_add(t0, kk * KSTEP), id_s, kk > 0);
#pragma unroll
        for (int kk = 0; kk < CH / 8; ++kk)
          tc::mma_tf32_ta(tm + T_DW, tm + T_AK + kk * 8, tc::desc_add(t0, kk * KSTEP), id_s, kk > 0);
        tc::mma_commit(&mbar);
      }
      ok = warp != 0 || tc::mbar_wait(&mbar, 1);
      if (__syncthreads_or(!ok)) {
        if (tid == 0) report(p.status, WKVM_ERR_TIMEOUT);
        tc::mbar_wait(&mbar, 1);
        break;
      }
      tc::fence_after_sync();
      {
        const int t0 = gh * 32;
        float x[32];
        tc::tmem_ld32(tq + T_D1 + t0, x);  // U^T[v = l][t0 + i] -> U[t][v], 128 B per warp and t
        __half* ucol = reinterpret_cast<__half*>(rec + R_U) + (l >> 6) * 64 * 64 + (l & 63);
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          ucol[(t0 + i) * 64] = __float2half_rn(x[i]);
          rmax = fmaxf(rmax, fabsf(x[i]));
        }
        // W^T[k = l][t0 + i] -> row-major W[t][k] in the spent stage (row
        // stride W_ROW: lanes hit distinct banks), copied out below
        tc::tmem_ld32(tq + T_DW + t0, x);
        float* wst = reinterpret_cast<float*>(sg);
#pragma unroll
        for (int i = 0; i < 32; ++i) wst[(t0 + i) * W_ROW + l] = x[i];
        if (tid == 0) *reinterpret_cast<float*>(rec + R_META) = __expf(GC);
      }
      __syncthreads();
      {  // W -> the record's K-major [W] rows: eight lanes fill one 128-byte core
         // matrix row group, a warp 512 contiguous bytes
        const float* wst = reinterpret_cast<const float*>(sg);
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          const int e = tid + WY_THREADS * jj;
          const int t = (e >> 7) * 8 + (e & 7), k8 = ((e >> 3) & 15) * 8;
          float wv[8];
          *reinterpret_cast<float4*>(wv) = *reinterpret_cast<const float4*>(wst + t * W_ROW + k8);
          *reinterpret_cast<float4*>(wv + 4) =
              *reinterpret_cast<const float4*>(wst + t * W_ROW + k8 + 4);
          st_h8(rec + R_WQ + hoff16(t, k8, SBOH128), wv, rmax);
        }
      }
      // the next job overwrites this stage only after every thread is past here
      tc::fence_before_sync();
      __syncthreads();
      tc::fence_after_sync();
    }
    cur = nxt;
#pragma unroll
    for (int i = 0; i < 4; ++i) sc_cur[i] = sc_next[i];
  }

  if (!(rmax <= kHalfMax)) report(p.status, WKVM_ERR_UNSUPPORTED);  // also NaN
  // no TMA load may still target this CTA's shared memory
  for (int st = 0; st < 2; ++st)
    if (((in_pending >> st) & 1u) && warp == 0 &&
        !tc::mbar_wait(&in_bar[st], (in_phase >> st) & 1u) && lane == 0)
      report(p.status, WKVM_ERR_TIMEOUT);
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tm, WY_TMEM_COLS);
}

// ---------------------------------------------------------------- phase 2

// Two CTAs per (sequence, value head): CTA vh owns value columns
// [64 vh, 64 vh + 64), so a sequence-head's chain runs on two SMs and each
// CTA issues M = 64 MMAs. An M = 64 tile occupies TMEM lanes 0..15 of each
// 32-lane quarter (row r at lane 32 (r / 16) + r % 16), for accumulators and
// for A operands alike, so lanes 16..31 of every warp carry no data.
// Warp roles: warps 0..7 (two per TMEM lane quarter) form u, rescale S,
// refresh the fp16 copy of S^T and write the outputs; warp 8 issues every
// copy and MMA and waits on the mbarriers that gate them. The two sides meet
// only on mbarriers, so the chain per chunk is MMA A -> u pass -> MMA B ->
// fp16 copy of S^T, with no CTA-wide barrier. Both MMAs are kind::f16 (fp16
// operands, the tf32 significand; fp32 accumulation): S^T itself stays fp32
// in TMEM and the MMAs read its fp16 copy.
constexpr int ST_WORKERS = 256;
constexpr int ST_THREADS = ST_WORKERS + 32;
constexpr uint32_t SS_A0 = 0, SS_A1 = PART_A, SS_B = 2 * PART_A, SS_U = SS_B + PART_B;
constexpr uint32_t SS_M = SS_U + PART_U;  // e^(G_C)
constexpr uint32_t ST_SMEM = SS_M + 128 + 1024;
static_assert(ST_SMEM <= 227 * 1024, "shared memory budget");
// TMEM: S^T half (fp32, 128 columns), its fp16 copy (two k per column: A of
// MMA A), u^T in fp16 (A of MMA B), two MMA A accumulators
constexpr uint32_t ST_TMEM_COLS = 512;
constexpr uint32_t T_S = 0, T_S16 = 128, T_U16 = 192, T_DA0 = 256, T_DA1 = 384;

// 32 floats as 16 columns of fp16 pairs (element 2c in the low half).
__device__ __forceinline__ void pack_h16(const float (&x)[32], float (&y)[16]) {
#pragma unroll
  for (int c = 0; c < 16; ++c) {
    __half2 h = __floats2half2_rn(x[2 * c], x[2 * c + 1]);
    y[c] = *reinterpret_cast<float*>(&h);
  }
}

template <typename Tin>
__global__ void __launch_bounds__(ST_THREADS, 1) gdn_state_kernel(StateArgs p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024(smem_raw);
  // copies: [W; Q~] x2, K~ / A_qk, U; MMA A done, MMA B done, u pass done
  __shared__ uint64_t mb_a[2], mb_b, mb_u, mb_ma, mb_mb, mb_w, mb_c;
  __shared__ uint32_t tmem_slot;
  __shared__ int s_fail;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bool issuer_warp = warp == ST_WORKERS / 32;
  const bool live = lane < 16 && !issuer_warp;  // a lane of the M = 64 tile
  const int vl = (warp & 3) * 16 + (lane & 15);    // value column within the half
  const int gq = (warp >> 2) & 1;                  // which half of t / k this thread takes
  const int n = blockIdx.x, hv = blockIdx.y, vh = blockIdx.z;
  const int v = vh * 64 + vl;
  const int HV = p.HV;
  int64_t row = n;
  if (p.ids) {
    const int32_t id = p.ids[n];
    if (id < 0 || (int64_t)id >= p.num_slots) {
      if (tid == 0 && vh == 0) report(p.status, WKVM_ERR_SLOT_RANGE);
      return;
    }
    row = id;
  }
  const int64_t soff = ((p.src_slots ? row : n) * HV + hv) * (int64_t)(KD * VD);
  const int64_t doff = ((p.dst_slots ? row : n) * HV + hv) * (int64_t)(KD * VD);
  int64_t bos, len;
  if (p.cu) {
    bos = p.cu[n];
    len = p.cu[n + 1] - bos;
  } else {
    bos = (int64_t)n * p.T;
    len = p.T;
  }
  const int nch = (int)((len + CH - 1) / CH);
  const int cend = nch < p.w0 + p.W ? nch : p.w0 + p.W;
  const int cnt = cend - p.w0;
  const bool same = p.h_src == p.h_dst && soff == doff;
  if (cnt <= 0) {  // nothing in this window: carry this half of the state over
    if (p.h_dst && !same)
      for (int e = tid; e < KD * 64; e += ST_THREADS) {
        const int64_t o = (e >> 6) * VD + vh * 64 + (e & 63);
        p.h_dst[doff + o] = p.h_src ? p.h_src[soff + o] : 0.f;
      }
    return;
  }
  const uint8_t* recs = p.ws + ((int64_t)n * p.W * HV + hv) * (int64_t)REC_BYTES;
  const int64_t rstride = (int64_t)HV * REC_BYTES;  // between consecutive chunks
  Tin* __restrict__ go = static_cast<Tin*>(p.o);

  if (warp == 0) {
    tc::tmem_alloc(&tmem_slot, ST_TMEM_COLS);
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    tc::mbar_init(&mb_a[0], 1);
    tc::mbar_init(&mb_a[1], 1);
    tc::mbar_init(&mb_b, 1);
    tc::mbar_init(&mb_u, 1);
    tc::mbar_init(&mb_ma, 1);
    tc::mbar_init(&mb_mb, 1);
    tc::mbar_init(&mb_w, ST_WORKERS / 32);
    tc::mbar_init(&mb_c, ST_WORKERS / 32);
    tc::fence_mbar_init();
    s_fail = 0;
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tm = tmem_slot;
  const uint32_t tq = tc::tmem_addr(tm, (warp & 3) * 32, 0);

  // S^T[v][k] = h[k][v] for this half's v, and its fp16 copy
  if (!issuer_warp) {
#pragma unroll 1
    for (int kb = gq * 64; kb < gq * 64 + 64; kb += 32) {
      float x[32], y[16];
#pragma unroll
      for (int i = 0; i < 32; ++i)
        x[i] = (live && p.h_src) ? p.h_src[soff + (kb + i) * VD + v] : 0.f;
      tc::tmem_st32(tq + T_S + kb, x);
      pack_h16(x, y);
      tc::tmem_st16(tq + T_S16 + kb / 2, y);
    }
    tc::tmem_st_wait();
  }
  // the whole of S^T is in TMEM before the first MMA
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();

  if (issuer_warp) {
    if (lane == 0) {
      uint32_t ph_a[2] = {0, 0}, ph = 0;  // ph: the per-chunk barriers' parity
      int pend_a[2] = {0, 0}, pend_b = 0, pend_u = 0, pend_m = 0;
      auto issue_a = [&](int i) {
        const int b = i & 1;
        tc::mbar_expect_tx(&mb_a[b], PART_A);
        tc::bulk_g2s(sm + (b ? SS_A1 : SS_A0), recs + i * rstride + R_WQ, PART_A, &mb_a[b]);
        pend_a[b] = 1;
      };
      auto issue_b = [&](int i) {
        tc::mbar_expect_tx(&mb_b, PART_B);
        tc::bulk_g2s(sm + SS_B, recs + i * rstride + R_KT, PART_B, &mb_b);
        pend_b = 1;
      };
      auto issue_u = [&](int i) {  // this half of U, and e^(G_C)
        tc::mbar_expect_tx(&mb_u, PART_U + 16);
        tc::bulk_g2s(sm + SS_U, recs + i * rstride + R_U + vh * PART_U, PART_U, &mb_u);
        tc::bulk_g2s(sm + SS_M, recs + i * rstride + R_META, 16, &mb_u);
        pend_u = 1;
      };
      issue_a(0);
      issue_u(0);
      issue_b(0);
      if (cnt > 1) issue_a(1);
      const uint32_t id_a = tc::idesc_f16(64, 128, false), id_o = tc::idesc_f16(64, 64, false);
      bool ok = true;
#pragma unroll 1
      for (int i = 0; i < cnt && ok; ++i) {
        const int b = i & 1;
        const uint32_t da = b ? T_DA1 : T_DA0;
        // MMA A: S^T x [W; Q~]^T, once this chunk's [W; Q~] landed (the fp16
        // copy of S^T is current: the workers refreshed it after MMA B)
        if (!(ok = tc::mbar_wait(&mb_a[b], ph_a[b]))) break;
        ph_a[b] ^= 1u;
        pend_a[b] = 0;
        tc::fence_after_sync();
        {
          const uint64_t a0 = tc::smem_desc(tc::smem_u32(sm + (b ? SS_A1 : SS_A0)), LBO, SBOH128);
#pragma unroll
          for (int kk = 0; kk < KD / 16; ++kk)
            tc::mma_f16_ta(tm + da, tm + T_S16 + kk * 8, tc::desc_add(a0, kk * KSTEP16), id_a,
                           kk > 0);
          tc::mma_commit(&mb_ma);
          pend_m = 1;
        }
        // the u pass is done (MMA A read this buffer of [W; Q~], the
        // workers read U); MMA B: S^T += u^T K~ ; O^T += u^T A_qk^T, once
        // K~ / A_qk landed
        if (!(ok = tc::mbar_wait(&mb_w, ph))) break;
        pend_m = 0;  // the workers saw MMA A complete
        tc::fence_after_sync();
        if (!(ok = tc::mbar_wait(&mb_b, ph))) break;
        pend_b = 0;
        {
          const uint64_t k0 = tc::smem_desc(tc::smem_u32(sm + SS_B), LBO, SBOH64);
          const uint64_t q0 = tc::desc_add(k0, R_AQK - R_KT);
#pragma unroll
          for (int kk = 0; kk < CH / 16; ++kk)
            tc::mma_f16_ta(tm + T_S, tm + T_U16 + kk * 8, tc::desc_add(k0, kk * KSTEP16), id_a,
                           true);
#pragma unroll
          for (int kk = 0; kk < CH / 16; ++kk)
            tc::mma_f16_ta(tm + da + 64, tm + T_U16 + kk * 8, tc::desc_add(q0, kk * KSTEP16),
                           id_o, true);
          tc::mma_commit(&mb_mb);
          pend_m = 1;
        }
        // while MMA B runs: chunk i+2's [W; Q~] into the buffer MMA A read,
        // chunk i+1's U into the one the u pass read
        if (i + 2 < cnt) issue_a(i + 2);
        if (i + 1 < cnt) issue_u(i + 1);
        // the workers saw MMA B complete and refreshed the fp16 S^T
        if (!(ok = tc::mbar_wait(&mb_c, ph))) break;
        pend_m = 0;
        tc::fence_after_sync();
        ph ^= 1u;
        if (i + 1 < cnt) issue_b(i + 1);  // MMA B has read K~ / A_qk
      }
      if (!ok) {
        atomicExch(&s_fail, 1);
        report(p.status, WKVM_ERR_TIMEOUT);
        // let copies and MMAs in flight land before the shared memory goes away
        if (pend_a[0]) tc::mbar_wait(&mb_a[0], ph_a[0]);
        if (pend_a[1]) tc::mbar_wait(&mb_a[1], ph_a[1]);
        if (pend_b) tc::mbar_wait(&mb_b, ph);
        if (pend_u) tc::mbar_wait(&mb_u, ph);
        if (pend_m) {
          tc::mbar_wait(&mb_ma, ph);
          tc::mbar_wait(&mb_mb, ph);
        }
      }
    }
    __syncwarp();
  } else {
    // O^T of chunk i (accumulator da) -> o rows t in this thread's half.
    // Lane pairs swap values so that each store writes two adjacent
    // columns: the even lane takes rows t0 .. t0+15, the odd lane t0+16 ..
    auto output = [&](int i, uint32_t da) {
      const int c = p.w0 + i;
      const int64_t tok0 = bos + (int64_t)c * CH;
      const int clen = (len - (int64_t)c * CH) < CH ? (int)(len - (int64_t)c * CH) : CH;
      const int t0 = gq * 32;
      float x[32];
      tc::tmem_ld32(tq + da + 64 + t0, x);
      const bool odd = lane & 1;
      Tin* col = go + (tok0 * HV + hv) * VD + (v & ~1);
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const float mine = odd ? x[j + 16] : x[j];
        const float give = odd ? x[j] : x[j + 16];
        const float other = __shfl_xor_sync(0xffffffffu, give, 1);
        const int t = t0 + j + (odd ? 16 : 0);
        union { uint32_t u; Tin e[2]; } pk;
        pk.e[0] = from_f32<Tin>(odd ? other : mine);
        pk.e[1] = from_f32<Tin>(odd ? mine : other);
        if (live && t < clen) *reinterpret_cast<uint32_t*>(col + (int64_t)t * HV * VD) = pk.u;
      }
    };
    // lane 0 polls a barrier, the warp follows; false once the issuer gave up
    auto wait_warp = [&](uint64_t* mb, uint32_t ph) -> bool {
      bool ok = true;
      if (lane == 0) {
        for (;;) {
          if (tc::mbar_wait(mb, ph, 1u << 12)) break;
          if (*static_cast<volatile int*>(&s_fail) || !(ok = tc::mbar_wait(mb, ph))) {
            ok = false;
            break;
          }
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      tc::fence_after_sync();
      return ok;
    };
    uint32_t ph = 0;
#pragma unroll 1
    for (int i = 0; i < cnt; ++i) {
      const uint32_t da = (i & 1) ? T_DA1 : T_DA0;
      if (!wait_warp(&mb_ma, ph) || !wait_warp(&mb_u, ph)) break;
      {  // u^T = U^T - (W S)^T in fp16 ; S^T *= e^(G_C)
        const __half* ucol = reinterpret_cast<const __half*>(sm + SS_U) + vl;
        const int t0 = gq * 32;
        float x[32], y[16];
        tc::tmem_ld32(tq + da + t0, x);
#pragma unroll
        for (int j = 0; j < 32; ++j) x[j] = __half2float(ucol[(t0 + j) * 64]) - x[j];
        pack_h16(x, y);
        tc::tmem_st16(tq + T_U16 + t0 / 2, y);
        const float eg = *reinterpret_cast<const float*>(sm + SS_M);
#pragma unroll 1
        for (int kb = gq * 64; kb < gq * 64 + 64; kb += 32) {
          float z[32];
          tc::tmem_ld32(tq + T_S + kb, z);
#pragma unroll
          for (int j = 0; j < 32; ++j) z[j] *= eg;
          tc::tmem_st32(tq + T_S + kb, z);
        }
        tc::tmem_st_wait();
      }
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&mb_w);
      // MMA B completes S^T for the next chunk (and O^T of this one): its
      // fp16 copy first, then the outputs, which overlap the next MMA A
      if (!wait_warp(&mb_mb, ph)) break;
#pragma unroll 1
      for (int kb = gq * 64; kb < gq * 64 + 64; kb += 32) {
        float z[32], y[16];
        tc::tmem_ld32(tq + T_S + kb, z);
        pack_h16(z, y);
        tc::tmem_st16(tq + T_S16 + kb / 2, y);
      }
      tc::tmem_st_wait();
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&mb_c);
      output(i, da);
      ph ^= 1u;
    }
    if (!*static_cast<volatile int*>(&s_fail) && p.h_dst) {
#pragma unroll 1
      for (int kb = gq * 64; kb < gq * 64 + 64; kb += 32) {
        float x[32];
        tc::tmem_ld32(tq + T_S + kb, x);
        if (live) {
#pragma unroll
          for (int i = 0; i < 32; ++i) p.h_dst[doff + (kb + i) * VD + v] = x[i];
        }
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tm, ST_TMEM_COLS);
}

template <typename Tin>
int run_windows(const WyArgs& wa0, const int32_t* ids, int64_t num_slots, const float* h_in, float* h_out, bool slots, float* carry,
                void* o, int nseq, int64_t max_chunks, int64_t W, cudaStream_t stream) {
  auto k1 = gdn_wy_kernel<Tin>;
  WyMaps maps;
  const int64_t tokens = wa0.cu ? (int64_t)wa0.T : (int64_t)nseq * wa0.T;
  if (tokens > 0) {
    int rc = tma::encode_rows(&maps.q, wa0.q, tokens, wa0.H, KD, CH);
    if (rc == WKVM_OK) rc = tma::encode_rows(&maps.k, wa0.k, tokens, wa0.H, KD, CH);
    if (rc == WKVM_OK) rc = tma::encode_rows(&maps.v, wa0.v, tokens, wa0.HV, VD, CH);
    if (rc != WKVM_OK) return rc;
  }
  auto k2 = gdn_state_kernel<Tin>;
  int dev = 0, num_sms = 148;
  WKVM_CUDA_TRY(cudaGetDevice(&dev));
  WKVM_CUDA_TRY(cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, dev));
  WKVM_CUDA_TRY(cudaFuncSetAttribute(k1, cudaFuncAttributeMaxDynamicSharedMemorySize, WY_SMEM));
  WKVM_CUDA_TRY(cudaFuncSetAttribute(k2, cudaFuncAttributeMaxDynamicSharedMemorySize, ST_SMEM));
  // one window: h_in -> h_out directly; several: h_in -> carry -> ... -> h_out
  const int64_t nwin = max_chunks > 0 ? (max_chunks + W - 1) / W : 1;
  for (int64_t w = 0; w < nwin; ++w) {
    WyArgs a = wa0;
    a.w0 = (int)(w * W);
    const int64_t wn = max_chunks - a.w0 < W ? max_chunks - a.w0 : W;
    const bool first = w == 0, final = w == nwin - 1;
    StateArgs sa{a.ws, o, first ? h_in : carry, final ? h_out : carry, first && slots,
                 final && slots, ids, num_slots, a.cu, a.T, a.HV, a.w0, (int)W, a.status};
    if (wn > 0) {
      const int njobs = (int)(wn * nseq * a.HV);
      const int grid = njobs < 2 * num_sms ? njobs : 2 * num_sms;
      k1<<<grid, WY_THREADS, WY_SMEM, stream>>>(a, njobs, maps);
    }
    k2<<<dim3(nseq, a.HV, 2), ST_THREADS, ST_SMEM, stream>>>(sa);
    WKVM_CUDA_TRY(cudaGetLastError());
  }
  return WKVM_OK;
}

}  // namespace

int64_t gdn_two_phase_workspace_bytes(int64_t nseq, int64_t T, int64_t HV) {
  const int64_t chunks = (T + gdnwy::CH - 1) / gdnwy::CH;
  return chunks * nseq * HV * (int64_t)gdnwy::REC_BYTES;
}

// Runs the two-phase prefill when the workspace holds at least one window;
// returns WKVM_ERR_UNSUPPORTED otherwise (the caller then runs the one-kernel
// path). h_in / h_out are indexed by slot id when `slots` is set.
int gdn_two_phase(const void* q, const void* k, const void* v, const void* g, const void* beta,
                  void* o, const float* h_in, float* h_out, bool slots, const int32_t* ids,
                  int64_t num_slots, const int64_t* cu, int nseq, int T, int H, int HV,
                  float scale, bool l2norm, int dtype, void* workspace, int64_t ws_bytes,
                  int* status, cudaStream_t stream) {
  if (!workspace || (reinterpret_cast<uintptr_t>(workspace) & 255u)) return WKVM_ERR_UNSUPPORTED;
  const int64_t max_chunks = (T + CH - 1) / CH;
  const int64_t per_chunk = (int64_t)nseq * HV * REC_BYTES;
  const int64_t state_bytes = (int64_t)nseq * HV * KD * VD * 4;
  int64_t W;
  uint8_t* recs = static_cast<uint8_t*>(workspace);
  float* carry = nullptr;
  if (ws_bytes >= max_chunks * per_chunk) {
    W = max_chunks > 0 ? max_chunks : 1;
  } else {
    const int64_t sb = (state_bytes + 255) & ~int64_t(255);
    W = (ws_bytes - sb) / per_chunk;
    if (W < 1) return WKVM_ERR_UNSUPPORTED;
    carry = reinterpret_cast<float*>(recs);
    recs += sb;
  }
  if (W > max_chunks && max_chunks > 0) W = max_chunks;
  if (W * nseq * HV > 0x7fffffff) W = 0x7fffffff / ((int64_t)nseq * HV);
  if (W < 1) return WKVM_ERR_UNSUPPORTED;
  if (nseq > 65535 || HV > 65535) return WKVM_ERR_UNSUPPORTED;
  WyArgs wa{q, k, v, g, beta, recs, cu, T, H, HV, 0, (int)W, nseq, scale, l2norm, status,
            (dtype & WKVM_GATES_F32) != 0};
  return (dtype & ~WKVM_GATES_F32) == WKVM_DTYPE_BF16
             ? run_windows<__nv_bfloat16>(wa, ids, num_slots, h_in, h_out, slots, carry, o, nseq,
                                         max_chunks, W, stream)
             : run_windows<__half>(wa, ids, num_slots, h_in, h_out, slots, carry, o, nseq,
                                   max_chunks, W, stream);
}

}  // namespace wkvm

extern "C" int64_t wkvm_gdn_chunk_workspace_bytes(int32_t nseq, int32_t T, int32_t HV, int32_t K,
                                                  int32_t V) {
  if (nseq < 0 || T < 0 || HV <= 0 || K != wkvm::gdnwy::KD || V != wkvm::gdnwy::VD) return 0;
  return wkvm::gdn_two_phase_workspace_bytes(nseq, T, HV);
}
