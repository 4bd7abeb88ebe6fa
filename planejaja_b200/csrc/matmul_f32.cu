// matmul_f32.cu -- dense f32 matmul with the reference operator's layout:
//   C[M x N] = A[M x K] . B[K x N], row-major, f32 accumulation.
// Reference: crates/nodestor-vulkan/shaders/matmul.comp:27-68 (16x16 shared
// tiles) and its CPU twin cpu_matmul_f32 (src/pipeline.rs:1256-1268).
//
// This is the unquantized (F32 weight) branch of the operator, not the
// quantized hot path: a 64x64 shared-memory tile with a 4x4 register block
// per thread.  Each output is accumulated over k in ascending order with
// fused multiply-adds.
#include "nsq_common.cuh"

namespace nsq {

constexpr int MT = 64, NT = 64, KT = 16;

__global__ void __launch_bounds__(256) matmul_f32_kernel(const float* __restrict__ A, const float* __restrict__ B,
                                                         float* __restrict__ C, int64_t M, int64_t K, int64_t N) {
  __shared__ float As[KT][MT + 4];
  __shared__ float Bs[KT][NT + 4];
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  const int64_t m0 = (int64_t)blockIdx.y * MT, n0 = (int64_t)blockIdx.x * NT;
  float acc[4][4] = {};
  for (int64_t k0 = 0; k0 < K; k0 += KT) {
    for (int i = threadIdx.x; i < MT * KT; i += 256) {
      const int r = i / KT, c = i % KT;
      const int64_t gm = m0 + r, gk = k0 + c;
      As[c][r] = (gm < M && gk < K) ? A[gm * K + gk] : 0.f;
    }
    for (int i = threadIdx.x; i < KT * NT; i += 256) {
      const int r = i / NT, c = i % NT;
      const int64_t gk = k0 + r, gn = n0 + c;
      Bs[r][c] = (gk < K && gn < N) ? B[gk * N + gn] : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < KT; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t gm = m0 + ty * 4 + i, gn = n0 + tx * 4 + j;
      if (gm < M && gn < N) C[gm * N + gn] = acc[i][j];
    }
}

cudaError_t launch_matmul_f32(const float* a, const float* b, float* c, int64_t M, int64_t K, int64_t N,
                              cudaStream_t st) {
  const int64_t gx = (N + NT - 1) / NT, gy = (M + MT - 1) / MT;
  if (gy > 65535) return cudaErrorInvalidValue;
  dim3 grid((unsigned)gx, (unsigned)gy);
  note_launch();
  matmul_f32_kernel<<<grid, 256, 0, st>>>(a, b, c, M, K, N);
  return cudaGetLastError();
}

}  // namespace nsq
