// The general GEMM kernel (simt family) and the alpha == 0 scale-C kernel.
//
// simt: 64 x 64 output tile per CTA, BK = 16, 256 threads with a 4 x 4 FP32
// micro-tile each, operands staged through shared memory as FP32 with
// element loads that honour any layout, leading dimension, batch stride and
// alignment. It is the path for problems the TMA tier cannot address
// (misaligned pointers or ld), the role of the reference's cp.async fallback
// (src/gemm/mma_pipe_impl.cuh:76-87 with mma_common.cuh:273-295). Out-of-range
// rows/columns/k are staged as zeros and never stored.
#include <algorithm>

#include "common.cuh"
#include "gpu_target.h"
#include "kernels.h"

namespace aegis {

using gemm::DType;
using gemm::GemmParams;
using gemm::Layout;

namespace {

constexpr int SB = 64, SBK = 16, SThreads = 256;

struct SimtArgs {
  const void* A;
  const void* B;
  void* C;
  int M, N, K;
  int ra, rb;  // row-major A / B
  long long lda, ldb, ldc, sa, sb, sc;
  float alpha, beta;
  int tiles_n;
  int batch0;  // first batch of this launch (blockIdx.z is relative)
};

template <class T>
__global__ void __launch_bounds__(SThreads) simt_gemm_kernel(SimtArgs a) {
  using E = Elem<T>;
  __shared__ float sA[SBK][SB + 4];
  __shared__ float sB[SBK][SB + 4];
  const int tid = int(threadIdx.x);
  const int tm = tid / 16, tn = tid % 16;
  const long long tile = blockIdx.x;
  const int m0 = int(tile / a.tiles_n) * SB, n0 = int(tile % a.tiles_n) * SB;
  const long long b = a.batch0 + blockIdx.z;
  const T* A = static_cast<const T*>(a.A) + b * a.sa;
  const T* B = static_cast<const T*>(a.B) + b * a.sb;
  T* C = static_cast<T*>(a.C) + b * a.sc;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < a.K; k0 += SBK) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int e = tid + i * SThreads;  // 0..1023
      // A: (m, k) = (e / 16, e % 16) for row-major (k fastest), (e % 64, e / 64) otherwise.
      int mm, kk;
      if (a.ra) { mm = e / SBK; kk = e % SBK; } else { mm = e % SB; kk = e / SB; }
      const int gm = m0 + mm, gk = k0 + kk;
      float v = 0.f;
      if (gm < a.M && gk < a.K) v = E::to_f32(a.ra ? A[(long long)gm * a.lda + gk] : A[gm + (long long)gk * a.lda]);
      sA[kk][mm] = v;
      // B: (k, n) = (e / 64, e % 64) for row-major (n fastest), (e % 16, e / 16) otherwise.
      int bk, bn;
      if (a.rb) { bk = e / SB; bn = e % SB; } else { bk = e % SBK; bn = e / SBK; }
      const int hk = k0 + bk, hn = n0 + bn;
      float w = 0.f;
      if (hk < a.K && hn < a.N) w = E::to_f32(a.rb ? B[(long long)hk * a.ldb + hn] : B[hk + (long long)hn * a.ldb]);
      sB[bk][bn] = w;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < SBK; ++kk) {
      float x[4], y[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) x[i] = sA[kk][tm * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) y[j] = sB[kk][tn * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(x[i], y[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int gm = m0 + tm * 4 + i;
    if (gm >= a.M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int gn = n0 + tn * 4 + j;
      if (gn >= a.N) continue;
      T* q = C + (long long)gm * a.ldc + gn;
      float v = a.alpha * acc[i][j];
      if (a.beta != 0.f) v += a.beta * E::to_f32(*q);
      *q = E::from_f32(v);
    }
  }
}

template <class T>
__global__ void __launch_bounds__(256) scale_c_kernel(T* C, int M, int N, long long ldc, long long stride_c,
                                                      int batch0, float beta) {
  using E = Elem<T>;
  T* c = C + (long long)(batch0 + blockIdx.z) * stride_c;
  const long long total = (long long)M * N;
  for (long long t = blockIdx.x * (long long)blockDim.x + threadIdx.x; t < total;
       t += (long long)gridDim.x * blockDim.x) {
    T* q = c + (t / N) * ldc + t % N;
    *q = E::from_f32(beta == 0.f ? 0.f : beta * E::to_f32(*q));
  }
}

constexpr int kMaxGridZ = 65535;

template <class T>
cudaError_t simt_launch(const GemmParams& p, cudaStream_t s) {
  SimtArgs a{};
  a.A = p.A;
  a.B = p.B;
  a.C = p.C;
  a.M = p.M;
  a.N = p.N;
  a.K = p.K;
  a.ra = p.layout_a == Layout::RowMajor;
  a.rb = p.layout_b == Layout::RowMajor;
  a.lda = p.lda;
  a.ldb = p.ldb;
  a.ldc = p.ldc;
  a.sa = p.stride_a;
  a.sb = p.stride_b;
  a.sc = p.stride_c;
  a.alpha = p.alpha;
  a.beta = p.beta;
  a.tiles_n = ceil_div(p.N, SB);
  const long long tiles = (long long)ceil_div(p.M, SB) * a.tiles_n;
  if (tiles > 0x7fffffffll) return cudaErrorInvalidConfiguration;
  for (int b0 = 0; b0 < p.batch; b0 += kMaxGridZ) {
    a.batch0 = b0;
    const int nb = std::min(kMaxGridZ, p.batch - b0);
    simt_gemm_kernel<T><<<dim3(unsigned(tiles), 1, unsigned(nb)), SThreads, 0, s>>>(a);
    if (const cudaError_t e = cudaGetLastError(); e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

template <class T>
cudaError_t scale_launch(const GemmParams& p, cudaStream_t s) {
  const long long total = (long long)p.M * p.N;
  const int blocks = int(std::min<long long>((total + 255) / 256, 1024));
  for (int b0 = 0; b0 < p.batch; b0 += kMaxGridZ) {
    const int nb = std::min(kMaxGridZ, p.batch - b0);
    scale_c_kernel<T><<<dim3(blocks, 1, nb), 256, 0, s>>>(static_cast<T*>(p.C), p.M, p.N, p.ldc, p.stride_c, b0,
                                                           p.beta);
    if (const cudaError_t e = cudaGetLastError(); e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace

cudaError_t simt_run(const GemmParams& p, cudaStream_t stream) {
  if (const cudaError_t e = gemm::validate(p); e != cudaSuccess) return e;
  if (gemm::is_empty(p)) return cudaSuccess;
  if (p.alpha == 0.f) return scale_c(p, stream);
  return p.dtype == DType::BF16 ? simt_launch<__nv_bfloat16>(p, stream) : simt_launch<__half>(p, stream);
}

cudaError_t scale_c(const GemmParams& p, cudaStream_t stream) {
  return p.dtype == DType::BF16 ? scale_launch<__nv_bfloat16>(p, stream) : scale_launch<__half>(p, stream);
}

cudaError_t simt_attrs(cudaFuncAttributes* attrs) { return cudaFuncGetAttributes(attrs, &simt_gemm_kernel<__half>); }

}  // namespace aegis
