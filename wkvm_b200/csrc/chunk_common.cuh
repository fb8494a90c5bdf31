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
  if (tid < 64) {  // diagonal 16 x 16 blocks, one column per thread
    const int col = tid, b0 = col & ~15, ci = col & 15;
    float y[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float* ar = Aab + (b0 + i) * RS + b0;
      float a[16];
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) {
        if (4 * q4 < i) {
          const float4 t4 = ld4(ar + 4 * q4);
          a[4 * q4] = t4.x;
          a[4 * q4 + 1] = t4.y;
          a[4 * q4 + 2] = t4.z;
          a[4 * q4 + 3] = t4.w;
        }
      }
      float v = (i == ci) ? 1.f : 0.f;
#pragma unroll
      for (int i2 = 0; i2 < i; ++i2) v = fmaf(a[i2], y[i2], v);
      y[i] = (i < ci) ? 0.f : v;
      Tr[(b0 + i) * RS + col] = y[i];
    }
    if (b0 & 16) {  // the 16-block above this diagonal block is zero
#pragma unroll
      for (int i = 0; i < 16; ++i) Tr[(b0 - 16 + i) * RS + col] = 0.f;
    }
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
