// Shared pieces of the chunked tensor-core prefill kernels (RWKV-7 DPLR and
// the gated delta rule): async staging copies, K-major tile stores and the
// blocked inverse of the 64 x 64 unit lower-triangular chunk matrix.
#pragma once

#include "tcgen05.cuh"

namespace wkvm {
namespace chunkc {

constexpr int RS = 68;  // row stride (floats) of row-major 64-wide scratch

__device__ __forceinline__ void kst4(uint8_t* tile, int row, int k, uint32_t lbo, uint32_t sbo,
                                     float4 x) {
  *reinterpret_cast<float4*>(tile + tc::kmajor_off(row, k, lbo, sbo)) = x;
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" :: "r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_group 0;" ::: "memory");
}

// T = (I - A)^-1 for a strictly lower-triangular 64 x 64 A (row-major, stride
// RS), blocked 16 -> 32 -> 64: the four diagonal 16-blocks by forward
// substitution, then T_ij = T_ii A_ij T_jj for the off-diagonal blocks.
// Written as a K-major tf32 operand tile (row t', K = t; LBO 128, SBO 2048),
// zero above the diagonal. Trow is row-major scratch (stride RS). With
// group == 0 every thread of the CTA (256 or more) calls it and threads 256
// and up only take part in the barriers; with group == 256 only threads
// 0..255 call it and synchronise on named barrier 1, so the other threads of
// the CTA can work meanwhile. Ends with the tile write, without a barrier
// (the caller fences and synchronises before the tensor core reads it).
__device__ __forceinline__ void group_sync(int group) {
  if (group == 0) __syncthreads();
  else asm volatile("bar.sync 1, %0;" :: "r"(group) : "memory");
}

__device__ __forceinline__ float4 ld4(const float* p) {
  return *reinterpret_cast<const float4*>(p);
}

// Rows of A and T are read as float4 (16-byte aligned: RS and every column
// offset used are multiples of 4), columns as scalars; the diagonal 16-blocks
// and the two upper 16-blocks the 32-merges read (rows 0..15 x cols 16..31,
// rows 32..47 x cols 48..63) are written with their zeros, so no product
// needs a mask.
__device__ __forceinline__ void tri_inverse64(const float* __restrict__ Aab, float* Trow,
                                              uint8_t* tt_tile, int tid, int group = 0) {
  float* Tr = Trow;
  const bool act = tid < 256;
  // ---- stage 1: the four diagonal 16 x 16 blocks, one warp each (warps 0..3,
  //      lane ln), blocked 4 -> 8 -> 16 with warp-level synchronisation; every
  //      block above a diagonal block that a later product reads is written as
  //      zero.
  if (act && tid < 128) {
    const int ln = tid & 31, blk = tid >> 5, b0 = blk * 16;
    if (ln < 16) {  // 4 x 4 diagonal blocks: column c of sub-block sb
      const int c = ln, sb = c >> 2, ci = c & 3, r0 = b0 + sb * 4;
      const float4 a1 = ld4(Aab + (r0 + 1) * RS + r0), a2 = ld4(Aab + (r0 + 2) * RS + r0),
                   a3 = ld4(Aab + (r0 + 3) * RS + r0);
      const float y0 = ci == 0 ? 1.f : 0.f;
      float y1 = fmaf(a1.x, y0, ci == 1 ? 1.f : 0.f);
      y1 = ci > 1 ? 0.f : y1;
      float y2 = fmaf(a2.y, y1, fmaf(a2.x, y0, ci == 2 ? 1.f : 0.f));
      y2 = ci > 2 ? 0.f : y2;
      const float y3 = fmaf(a3.z, y2, fmaf(a3.y, y1, fmaf(a3.x, y0, ci == 3 ? 1.f : 0.f)));
      float* tc0 = Tr + r0 * RS + b0 + c;
      tc0[0] = y0;
      tc0[RS] = y1;
      tc0[2 * RS] = y2;
      tc0[3 * RS] = y3;
      if (sb & 1) {  // the 4-block above is zero
#pragma unroll
        for (int i = 0; i < 4; ++i) tc0[(i - 4) * RS] = 0.f;
      }
      if (sb >= 2) {  // and the 8-block above, rows b0 .. b0+7
#pragma unroll
        for (int i = 0; i < 8; ++i) Tr[(b0 + i) * RS + b0 + c] = 0.f;
      }
      if (blk & 1) {  // and the 16-block above this diagonal block
#pragma unroll
        for (int i = 0; i < 16; ++i) Tr[(b0 - 16 + i) * RS + b0 + c] = 0.f;
      }
    }
    __syncwarp();
    // 4 -> 8: blocks (1,0) of each 8 x 8 diagonal block (m = 0, 1)
    const int m = ln >> 4, r = (ln >> 2) & 3, cc = ln & 3, e0 = b0 + 8 * m;
    {
      const float4 a4 = ld4(Aab + (e0 + 4 + r) * RS + e0);
      const float* tcol = Tr + e0 * RS + e0 + cc;
      const float xq = fmaf(a4.x, tcol[0], fmaf(a4.y, tcol[RS], fmaf(a4.z, tcol[2 * RS],
                            a4.w * tcol[3 * RS])));
      Tr[(e0 + 4 + r) * RS + e0 + cc] = xq;
    }
    __syncwarp();
    float yq;
    {
      const float4 t4 = ld4(Tr + (e0 + 4 + r) * RS + e0 + 4);
      const float* xc = Tr + (e0 + 4) * RS + e0 + cc;
      yq = fmaf(t4.x, xc[0], fmaf(t4.y, xc[RS], fmaf(t4.z, xc[2 * RS], t4.w * xc[3 * RS])));
    }
    __syncwarp();
    Tr[(e0 + 4 + r) * RS + e0 + cc] = yq;
    __syncwarp();
    // 8 -> 16: block (1,0) of the 16 x 16 diagonal block, X = A_10 T_00, T_10 = T_11 X;
    // lane: column c8, rows r8 and r8 + 4
    const int c8 = ln & 7, ra = ln >> 3;
    float x8[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r8 = ra + 4 * h;
      const float4 a0 = ld4(Aab + (b0 + 8 + r8) * RS + b0),
                   a1 = ld4(Aab + (b0 + 8 + r8) * RS + b0 + 4);
      const float* tcol = Tr + b0 * RS + b0 + c8;
      x8[h] = fmaf(a0.x, tcol[0], fmaf(a0.y, tcol[RS], fmaf(a0.z, tcol[2 * RS],
              fmaf(a0.w, tcol[3 * RS], fmaf(a1.x, tcol[4 * RS], fmaf(a1.y, tcol[5 * RS],
              fmaf(a1.z, tcol[6 * RS], a1.w * tcol[7 * RS])))))));
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) Tr[(b0 + 8 + ra + 4 * h) * RS + b0 + c8] = x8[h];
    __syncwarp();
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r8 = ra + 4 * h;
      const float4 t0 = ld4(Tr + (b0 + 8 + r8) * RS + b0 + 8),
                   t1 = ld4(Tr + (b0 + 8 + r8) * RS + b0 + 12);
      const float* xc = Tr + (b0 + 8) * RS + b0 + c8;
      x8[h] = fmaf(t0.x, xc[0], fmaf(t0.y, xc[RS], fmaf(t0.z, xc[2 * RS],
              fmaf(t0.w, xc[3 * RS], fmaf(t1.x, xc[4 * RS], fmaf(t1.y, xc[5 * RS],
              fmaf(t1.z, xc[6 * RS], t1.w * xc[7 * RS])))))));
    }
    __syncwarp();
#pragma unroll
    for (int h = 0; h < 2; ++h) Tr[(b0 + 8 + ra + 4 * h) * RS + b0 + c8] = x8[h];
  }
  group_sync(group);
  // blocks (1,0) and (3,2) of 16: X = A T_jj, then T_ij = T_ii X.
  // Thread: row r = (tid >> 4) & 15, column cc = tid & 15 of both blocks.
  const int r = (tid >> 4) & 15, cc = tid & 15;
  float xv[4] = {0.f, 0.f, 0.f, 0.f};
  if (act) {
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const float* ar = Aab + (32 * q + 16 + r) * RS + 32 * q;
      const float* tc0 = Tr + (32 * q) * RS + 32 * q + cc;
      float x = 0.f;
#pragma unroll
      for (int s4 = 0; s4 < 16; s4 += 4) {
        const float4 a4 = ld4(ar + s4);
        x = fmaf(a4.x, tc0[(s4 + 0) * RS], x);
        x = fmaf(a4.y, tc0[(s4 + 1) * RS], x);
        x = fmaf(a4.z, tc0[(s4 + 2) * RS], x);
        x = fmaf(a4.w, tc0[(s4 + 3) * RS], x);
      }
      xv[q] = x;
    }
#pragma unroll
    for (int q = 0; q < 2; ++q) Tr[(32 * q + 16 + r) * RS + 32 * q + cc] = xv[q];
  }
  group_sync(group);
  if (act) {
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const float* tr = Tr + (32 * q + 16 + r) * RS + 32 * q + 16;
      const float* xc = Tr + (32 * q + 16) * RS + 32 * q + cc;
      float y = 0.f;
#pragma unroll
      for (int s4 = 0; s4 < 16; s4 += 4) {
        const float4 t4 = ld4(tr + s4);
        y = fmaf(t4.x, xc[(s4 + 0) * RS], y);
        y = fmaf(t4.y, xc[(s4 + 1) * RS], y);
        y = fmaf(t4.z, xc[(s4 + 2) * RS], y);
        y = fmaf(t4.w, xc[(s4 + 3) * RS], y);
      }
      xv[2 + q] = y;
    }
  }
  group_sync(group);
  if (act) {
#pragma unroll
    for (int q = 0; q < 2; ++q) Tr[(32 * q + 16 + r) * RS + 32 * q + cc] = xv[2 + q];
  }
  group_sync(group);
  // block (1,0) of 32: X = A T_00, then T_10 = T_11 X. Thread: column
  // C = tid & 31, rows 32 + (tid >> 5) + 8 q.
  const int C = tid & 31, r0 = (tid >> 5) & 7;
  if (act) {
#pragma unroll
    for (int q = 0; q < 4; ++q) xv[q] = 0.f;
#pragma unroll
    for (int s4 = 0; s4 < 32; s4 += 4) {
      float tv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) tv[i] = Tr[(s4 + i) * RS + C];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float4 a4 = ld4(Aab + (32 + r0 + 8 * q) * RS + s4);
        xv[q] = fmaf(a4.x, tv[0], xv[q]);
        xv[q] = fmaf(a4.y, tv[1], xv[q]);
        xv[q] = fmaf(a4.z, tv[2], xv[q]);
        xv[q] = fmaf(a4.w, tv[3], xv[q]);
      }
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) Tr[(32 + r0 + 8 * q) * RS + C] = xv[q];
  }
  group_sync(group);
  if (act) {
    float yv[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int s4 = 0; s4 < 32; s4 += 4) {
      float xx[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) xx[i] = Tr[(32 + s4 + i) * RS + C];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float4 t4 = ld4(Tr + (32 + r0 + 8 * q) * RS + 32 + s4);
        yv[q] = fmaf(t4.x, xx[0], yv[q]);
        yv[q] = fmaf(t4.y, xx[1], yv[q]);
        yv[q] = fmaf(t4.z, xx[2], yv[q]);
        yv[q] = fmaf(t4.w, xx[3], yv[q]);
      }
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) xv[q] = yv[q];
  }
  group_sync(group);
  if (act) {
#pragma unroll
    for (int q = 0; q < 4; ++q) Tr[(32 + r0 + 8 * q) * RS + C] = xv[q];
  }
  group_sync(group);
  if (act) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {  // K-major tile, zero above the diagonal;
      // lanes walk 8 rows x 4 K-quads so each store instruction fills 512
      // contiguous bytes
      const int e = tid + 256 * q;
      const int tp = (e >> 7) * 8 + (e & 7), t4 = ((e >> 3) & 15) * 4;
      float v4[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) v4[i] = (t4 + i <= tp) ? Tr[tp * RS + t4 + i] : 0.f;
      kst4(tt_tile, tp, t4, 128u, 2048u, make_float4(v4[0], v4[1], v4[2], v4[3]));
    }
  }
}

}  // namespace chunkc
}  // namespace wkvm
