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

__device__ __forceinline__ void tri_inverse64(const float* __restrict__ Aab, float* Trow,
                                              uint8_t* tt_tile, int tid, int group = 0) {
  float* Tr = Trow;
  const bool act = tid < 256;
  if (tid < 64) {  // diagonal 16 x 16 blocks, one column per thread
    const int col = tid, b0 = col & ~15, ci = col & 15;
    float y[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      float v = (i == ci) ? 1.f : 0.f;
#pragma unroll
      for (int i2 = 0; i2 < i; ++i2) v = fmaf(Aab[(b0 + i) * RS + b0 + i2], y[i2], v);
      y[i] = (i < ci) ? 0.f : v;
      Tr[(b0 + i) * RS + col] = y[i];
    }
  }
  group_sync(group);
  // blocks (1,0) and (3,2) of 16: X = A T_jj, then T_ij = T_ii X.
  // Thread: row r = (tid >> 4) & 15, column cc = tid & 15 of both blocks.
  const int r = (tid >> 4) & 15, cc = tid & 15;
  float xv[4] = {0.f, 0.f, 0.f, 0.f};
  if (act) {
#pragma unroll
    for (int s2 = 0; s2 < 16; ++s2) {
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const float tv = Tr[(32 * q + s2) * RS + 32 * q + cc];
        const float av = Aab[(32 * q + 16 + r) * RS + 32 * q + s2];
        xv[q] = fmaf(av, s2 >= cc ? tv : 0.f, xv[q]);
      }
    }
#pragma unroll
    for (int q = 0; q < 2; ++q) Tr[(32 * q + 16 + r) * RS + 32 * q + cc] = xv[q];
  }
  group_sync(group);
  if (act) {
    float yv[2] = {0.f, 0.f};
#pragma unroll
    for (int s2 = 0; s2 < 16; ++s2) {
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const float tv = Tr[(32 * q + 16 + r) * RS + 32 * q + 16 + s2];
        const float xx = Tr[(32 * q + 16 + s2) * RS + 32 * q + cc];
        yv[q] = fmaf(s2 <= r ? tv : 0.f, xx, yv[q]);
      }
    }
    xv[0] = yv[0];
    xv[1] = yv[1];
  }
  group_sync(group);
  if (act) {
#pragma unroll
    for (int q = 0; q < 2; ++q) Tr[(32 * q + 16 + r) * RS + 32 * q + cc] = xv[q];
  }
  group_sync(group);
  // block (1,0) of 32: X = A T_00, then T_10 = T_11 X. Thread: column
  // C = tid & 31, rows 32 + (tid >> 5) + 8 q.
  const int C = tid & 31, r0 = (tid >> 5) & 7;
  if (act) {
#pragma unroll
    for (int q = 0; q < 4; ++q) xv[q] = 0.f;
#pragma unroll
    for (int s2 = 0; s2 < 32; ++s2) {
      const float tv = s2 >= C ? Tr[s2 * RS + C] : 0.f;
#pragma unroll
      for (int q = 0; q < 4; ++q) xv[q] = fmaf(Aab[(32 + r0 + 8 * q) * RS + s2], tv, xv[q]);
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) Tr[(32 + r0 + 8 * q) * RS + C] = xv[q];
  }
  group_sync(group);
  if (act) {
    float yv[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int s2 = 0; s2 < 32; ++s2) {
      const float xx = Tr[(32 + s2) * RS + C];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int R = r0 + 8 * q;
        yv[q] = fmaf(s2 <= R ? Tr[(32 + R) * RS + 32 + s2] : 0.f, xx, yv[q]);
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
