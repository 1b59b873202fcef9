// Affine state combine for context-parallel prefill: out[h] = S[h] M[h] + N[h]
// for 128 x 128 fp32 matrices (k-last states, row = v).
//
// Over one segment of a sequence the chunked recurrence maps every state row
// the same affine way: S_end[v, :] = S_0[v, :] M + N[v, :], with M the product
// of the per-chunk maps e^{gamma_last} I - W^T K_decay and N the final state of
// a zero-state run (ref solution/cuda/kernel_prefill.cu:286-293 gives the
// per-chunk update this composes).  A rank of a context-parallel prefill
// learns its initial state by folding the maps of the segments before it
// through this kernel.  The work is tiny (2 * 128^3 flop per head), so it runs
// on CUDA cores in fp32: each CTA owns a 32 x 32 output tile of one head and
// walks k in 32-wide slabs staged in shared memory.
#pragma once

#include "decode_kernel.cuh"

namespace gdn {

constexpr int kAffineTile = 32;
constexpr int kAffineThreads = 256;   // 32 x 32 outputs, 4 per thread

__global__ void __launch_bounds__(kAffineThreads)
    gdn_state_affine_kernel(const float* __restrict__ S, const float* __restrict__ M,
                            const float* __restrict__ N, float* __restrict__ out) {
  __shared__ float sS[kAffineTile][kAffineTile + 1];
  __shared__ float sM[kAffineTile][kAffineTile + 1];
  const int h = blockIdx.y;
  const int tr = blockIdx.x / (kHeadDim / kAffineTile), tc = blockIdx.x % (kHeadDim / kAffineTile);
  const size_t base = static_cast<size_t>(h) * kHeadDim * kHeadDim;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;   // column, row group (8 rows)
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  if (S) {
    for (int k0 = 0; k0 < kHeadDim; k0 += kAffineTile) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = ty + 8 * i;
        sS[r][tx] = S[base + static_cast<size_t>(tr * kAffineTile + r) * kHeadDim + k0 + tx];
        sM[r][tx] = M[base + static_cast<size_t>(k0 + r) * kHeadDim + tc * kAffineTile + tx];
      }
      __syncthreads();
#pragma unroll 8
      for (int kk = 0; kk < kAffineTile; ++kk) {
        const float m = sM[kk][tx];
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[i] = fmaf(sS[ty + 8 * i][kk], m, acc[i]);
      }
      __syncthreads();
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const size_t o = base + static_cast<size_t>(tr * kAffineTile + ty + 8 * i) * kHeadDim +
                     tc * kAffineTile + tx;
    out[o] = acc[i] + N[o];
  }
}

}  // namespace gdn
