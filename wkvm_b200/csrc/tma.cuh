// Tensor Memory Accelerator (TMA) tile loads of activation rows, for the
// chunked prefill kernels (sm_100a).
//
// An activation tensor [tokens, heads, D] of 16-bit elements (fla's
// [B, T, H, D] with B*T flattened, or varlen [1, total, H, D]) is described
// to the TMA as a 3-D tensor (D, heads, tokens). One load brings a box of
// `rows` consecutive tokens of one head -- rows x D elements -- into shared
// memory with the 128-byte swizzle, completing on an mbarrier as transaction
// bytes. No multicast: every load reads this GPU's own input buffers into
// the issuing CTA's shared memory.
//
// The 128-byte swizzle stores row t of a box at t * 128 bytes, with its
// 16-byte pieces permuted: piece j lands at piece j ^ (t & 7). Readers go
// through sw128_off(). Rows beyond the tensor's last token arrive zero;
// rows past a sequence's end that still lie inside the tensor arrive with
// the next sequence's data and must be masked by the kernel.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace wkvm {
namespace tma {

// Byte offset of element byte `b` of row `t` in a 128-byte-swizzled box of
// 128-byte rows.
__device__ __forceinline__ uint32_t sw128_off(int t, uint32_t b) {
  return (uint32_t)t * 128u + ((((b >> 4) ^ (uint32_t)t) & 7u) << 4) + (b & 15u);
}

// 3-D tiled load (no multicast) of box {64, 1, rows} at (col0, head,
// token0) into `dst` (1024-byte aligned), counted on `mbar`. col0 is a
// multiple of 64 elements (128 bytes), so the box starts 16-byte aligned.
__device__ __forceinline__ void load_rows(void* dst, const CUtensorMap* map, int head, int token0,
                                          uint64_t* mbar, int col0 = 0) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];"
      :: "r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(reinterpret_cast<uint64_t>(map)),
         "r"(col0), "r"(head), "r"(token0), "r"((uint32_t)__cvta_generic_to_shared(mbar))
      : "memory");
}

__device__ __forceinline__ void prefetch_map(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" :: "l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Host: describes a [tokens, heads, D] tensor of 16-bit elements (D a
// multiple of 64) for boxes of `rows` tokens x 64 elements of one head.
// Returns 0 on success.
int encode_rows(CUtensorMap* map, const void* base, int64_t tokens, int heads, int D, int rows);

}  // namespace tma
}  // namespace wkvm
