// Self-test of the tcgen05 layer: one 128 x N x 64 tf32 GEMM tile
// D = A B^T with B staged by threads into the K-major no-swizzle layout and
// A either there too or written into tensor memory with tcgen05.st,
// accumulated in TMEM and read back with tcgen05.ld. Exposed so the
// test suite can pin the descriptor encodings the prefill kernels rely on.
#include "tcgen05.cuh"

namespace wkvm {
namespace {

constexpr uint32_t kLbo = 128;   // K-adjacent core matrices
constexpr uint32_t kSbo = 2048;  // 8-row groups (16 core matrices of K = 64)

__global__ void __launch_bounds__(128) tf32_mma_selftest_kernel(const float* __restrict__ A,
                                                                const float* __restrict__ B,
                                                                float* __restrict__ D, int N,
                                                                int a_in_tmem, int* status) {
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ uint64_t mbar;
  __shared__ uint32_t tmem_base;
  uint8_t* sA = smem;
  uint8_t* sB = smem + 128 * 64 * 4;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  for (int e = tid; e < 128 * 64; e += 128)
    *reinterpret_cast<float*>(sA + tc::kmajor_off(e >> 6, e & 63, kLbo, kSbo)) = A[e];
  for (int e = tid; e < N * 64; e += 128)
    *reinterpret_cast<float*>(sB + tc::kmajor_off(e >> 6, e & 63, kLbo, kSbo)) = B[e];
  if (warp == 0) {
    tc::tmem_alloc(&tmem_base, 256);
    tc::tmem_relinquish();
  }
  if (tid == 0) tc::mbar_init(&mbar, 1);
  tc::fence_smem_to_async();
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tbase = tmem_base;
  if (a_in_tmem) {
    // A row (warp*32 + lane) -> TMEM lane of this thread, columns [128, 192)
    for (int c = 0; c < 64; c += 32) {
      float v[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = A[(warp * 32 + lane) * 64 + c + i];
      tc::tmem_st32(tc::tmem_addr(tbase, warp * 32, 128 + c), v);
    }
    tc::tmem_st_wait();
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
  }

  if (tid == 0) {
    const uint32_t idesc = tc::idesc_tf32(128, N);
    for (int kk = 0; kk < 8; ++kk) {  // K = 8 tf32 elements (32 bytes) per MMA
      const uint64_t bd = tc::smem_desc(tc::smem_u32(sB) + kk * 2 * kLbo, kLbo, kSbo);
      if (a_in_tmem) {
        tc::mma_tf32_ta(tbase, tbase + 128 + kk * 8, bd, idesc, kk > 0);
      } else {
        const uint64_t ad = tc::smem_desc(tc::smem_u32(sA) + kk * 2 * kLbo, kLbo, kSbo);
        tc::mma_tf32(tbase, ad, bd, idesc, kk > 0);
      }
    }
    tc::mma_commit(&mbar);
  }
  const bool ok = tc::mbar_wait(&mbar, 0);
  if (!ok && tid == 0) report(status, WKVM_ERR_TIMEOUT);
  tc::fence_after_sync();
  if (ok) {
    const int row = warp * 32 + lane;
    for (int c = 0; c < N; c += 32) {
      float v[32];
      tc::tmem_ld32(tc::tmem_addr(tbase, warp * 32, c), v);
#pragma unroll
      for (int i = 0; i < 32; ++i) D[row * N + c + i] = v[i];
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tbase, 256);
}

}  // namespace
}  // namespace wkvm

extern "C" int wkvm_selftest_tf32_mma(const float* A, const float* B, float* D, int32_t N,
                                      int32_t a_in_tmem, int32_t* status,
                                      wkvm_stream_t stream) {
  if (!A || !B || !D) return WKVM_ERR_INVALID_ARG;
  if (N != 64 && N != 128) return WKVM_ERR_SHAPE;
  const int smem = (128 + N) * 64 * 4;
  auto k = wkvm::tf32_mma_selftest_kernel;
  WKVM_CUDA_TRY(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  k<<<1, 128, smem, (cudaStream_t)stream>>>(A, B, D, N, a_in_tmem, status);
  return cudaGetLastError() == cudaSuccess ? WKVM_OK : WKVM_ERR_CUDA;
}
