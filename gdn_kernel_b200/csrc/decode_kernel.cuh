// GDN decode (T = 1): one fused, bandwidth-bound pass over the fp32 k-last
// state [B, H_v, V, K].
//
// Semantics follow the reference decode kernel (ref solution/cuda/kernel.cu:21-97):
//   g = exp(-exp(A_log) softplus(a + dt_bias)),  beta = sigmoid(b)
//   S <- g S;  delta = beta (v - S k);  S += delta k^T;  o = scale S q
// written per state row v (rows are independent in the k-last layout):
//   s = g S_v;  delta_v = beta (v_v - <s,k>);  S_v' = s + delta_v k;
//   o_v = scale (<s,q> + delta_v <k,q>)
//
// Layout on the SM: a CTA of 4 warps covers kRowsPerCta = 16 * kIters rows of
// one (batch, v-head) state.  Eight lanes share one 512-byte state row (each
// lane holds four float4 at columns 4*l8 + 32*j), so one warp instruction moves
// four full rows, fully coalesced, and the two row reductions are 3-level xor
// shuffles.  Each warp streams 4 * kIters rows through a register pipeline
// kPipe iterations deep, writing every row back in place.
#pragma once

#include "gdn_ptx.cuh"

namespace gdn {

constexpr int kHeadDim = 128;
constexpr int kDecodeThreads = 128;
#ifndef GDN_DECODE_ITERS
#define GDN_DECODE_ITERS 1   // 4 rows per warp per iteration
#endif
#ifndef GDN_DECODE_PIPE
#define GDN_DECODE_PIPE 1    // iterations of loads in flight ahead of the reduction
#endif
#ifndef GDN_DECODE_LDHINT
#define GDN_DECODE_LDHINT 1  // L1::no_allocate + L2::256B prefetch on state loads
#endif
constexpr int kDecodeIters = GDN_DECODE_ITERS;
constexpr int kDecodePipe = GDN_DECODE_PIPE;
constexpr int kDecodeRowsPerCta = 16 * kDecodeIters;
constexpr int kDecodeCtasPerHead = kHeadDim / kDecodeRowsPerCta;
static_assert(kHeadDim % kDecodeRowsPerCta == 0, "rows per CTA must divide 128");

struct DecodeParams {
  const __nv_bfloat16* q;        // [B, 1, H_qk, K]
  const __nv_bfloat16* k;        // [B, 1, H_qk, K]
  const __nv_bfloat16* v;        // [B, 1, H_v, V]
  const float* state;            // [B, H_v, V, K] or nullptr (zero state)
  const float* A_log;            // [H_v]
  const __nv_bfloat16* a;        // [B, 1, H_v]
  const float* dt_bias;          // [H_v]
  const __nv_bfloat16* b;        // [B, 1, H_v]
  float scale;
  __nv_bfloat16* out;            // [B, 1, H_v, V]
  float* new_state;              // [B, H_v, V, K], may alias state
  int h_qk;
  int h_v;
};

__device__ __forceinline__ float softplus20(float x) {
  return x > 20.0f ? x : log1pf(expf(x));
}

__device__ __forceinline__ float4 ld_state(const float* p) {
  float4 r;
#if GDN_DECODE_LDHINT
  asm volatile("ld.global.L1::no_allocate.L2::256B.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w)
               : "l"(p));
#else
  asm volatile("ld.global.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w)
               : "l"(p));
#endif
  return r;
}

__device__ __forceinline__ void st_state(float* p, float4 r) {
  asm volatile("st.global.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(p), "f"(r.x), "f"(r.y), "f"(r.z),
               "f"(r.w)
               : "memory");
}

__device__ __forceinline__ void load_bf16x4(const __nv_bfloat16* p, float* dst) {
  uint2 u = *reinterpret_cast<const uint2*>(p);
  __nv_bfloat162 lo = *reinterpret_cast<__nv_bfloat162*>(&u.x);
  __nv_bfloat162 hi = *reinterpret_cast<__nv_bfloat162*>(&u.y);
  float2 f0 = __bfloat1622float2(lo), f1 = __bfloat1622float2(hi);
  dst[0] = f0.x; dst[1] = f0.y; dst[2] = f1.x; dst[3] = f1.y;
}

template <bool kHasState>
__global__ void __launch_bounds__(kDecodeThreads) gdn_decode_kernel(DecodeParams p) {
  constexpr int kIters = kDecodeIters;
  constexpr int kPipe = kDecodePipe < kDecodeIters ? kDecodePipe : kDecodeIters;
  constexpr int kBuf = kPipe < kDecodeIters ? kPipe + 1 : kDecodeIters;
  const int bh = blockIdx.x / kDecodeCtasPerHead;   // batch * H_v + v-head
  const int rblk = blockIdx.x % kDecodeCtasPerHead;
  const int h = bh % p.h_v;
  const int bidx = bh / p.h_v;
  const int hq = h / (p.h_v / p.h_qk);       // GQA: v-head h reads qk-head h / (H_v/H_qk)
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int sub = lane >> 3;                 // row inside the warp's 4-row group
  const int l8 = lane & 7;                   // column slot inside the row

  // State loads first: they are independent of the gate and q/k loads and
  // carry the DRAM latency that everything else overlaps with.
  const size_t sbase = static_cast<size_t>(bh) * kHeadDim * kHeadDim;
  // iteration it touches row row0 + 4*it
  const int row0 = rblk * kDecodeRowsPerCta + warp * (4 * kIters) + sub;
  const float* src = kHasState ? p.state + sbase + static_cast<size_t>(row0) * kHeadDim + 4 * l8
                               : nullptr;
  float* dst = p.new_state + sbase + static_cast<size_t>(row0) * kHeadDim + 4 * l8;
  const __nv_bfloat16* vrow = p.v + static_cast<size_t>(bh) * kHeadDim;

  float4 buf[kBuf][4];
  if (kHasState) {
#pragma unroll
    for (int it = 0; it < kPipe; ++it)
#pragma unroll
      for (int j = 0; j < 4; ++j) buf[it % kBuf][j] = ld_state(src + it * 4 * kHeadDim + 32 * j);
  }

  // Gate and beta for this (batch, v-head) (ref kernel.cu:44-53).
  const float av = __bfloat162float(p.a[bh]);
  const float bv = __bfloat162float(p.b[bh]);
  const float g = expf(-expf(p.A_log[h]) * softplus20(av + p.dt_bias[h]));
  const float beta = 1.0f / (1.0f + expf(-bv));

  // q and k fragments for columns 4*l8 + 32*j + e.
  const size_t qk_off = (static_cast<size_t>(bidx) * p.h_qk + hq) * kHeadDim;
  float qf[16], kf[16];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    load_bf16x4(p.q + qk_off + 4 * l8 + 32 * j, qf + 4 * j);
    load_bf16x4(p.k + qk_off + 4 * l8 + 32 * j, kf + 4 * j);
  }
  float qk = 0.f;
#pragma unroll
  for (int e = 0; e < 16; ++e) qk = fmaf(qf[e], kf[e], qk);
  qk += __shfl_xor_sync(0xffffffffu, qk, 1);
  qk += __shfl_xor_sync(0xffffffffu, qk, 2);
  qk += __shfl_xor_sync(0xffffffffu, qk, 4);

  float outv[kIters];
#pragma unroll
  for (int it = 0; it < kIters; ++it) {
    if (kHasState && it + kPipe < kIters) {
#pragma unroll
      for (int j = 0; j < 4; ++j)
        buf[(it + kPipe) % kBuf][j] = ld_state(src + (it + kPipe) * 4 * kHeadDim + 32 * j);
    }
    float s[16];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (kHasState) {
        const float4 x = buf[it % kBuf][j];
        s[4 * j + 0] = g * x.x; s[4 * j + 1] = g * x.y;
        s[4 * j + 2] = g * x.z; s[4 * j + 3] = g * x.w;
      } else {
        s[4 * j + 0] = s[4 * j + 1] = s[4 * j + 2] = s[4 * j + 3] = 0.f;
      }
    }
    float dk = 0.f, dq = 0.f;
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      dk = fmaf(s[e], kf[e], dk);
      dq = fmaf(s[e], qf[e], dq);
    }
#pragma unroll
    for (int m = 1; m < 8; m <<= 1) {
      dk += __shfl_xor_sync(0xffffffffu, dk, m);
      dq += __shfl_xor_sync(0xffffffffu, dq, m);
    }
    const float vv = __bfloat162float(vrow[row0 + 4 * it]);
    const float delta = beta * (vv - dk);
    outv[it] = p.scale * (dq + delta * qk);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float4 y;
      y.x = fmaf(delta, kf[4 * j + 0], s[4 * j + 0]);
      y.y = fmaf(delta, kf[4 * j + 1], s[4 * j + 1]);
      y.z = fmaf(delta, kf[4 * j + 2], s[4 * j + 2]);
      y.w = fmaf(delta, kf[4 * j + 3], s[4 * j + 3]);
      st_state(dst + it * 4 * kHeadDim + 32 * j, y);
    }
  }
  if (l8 == 0) {
    __nv_bfloat16* orow = p.out + static_cast<size_t>(bh) * kHeadDim;
#pragma unroll
    for (int it = 0; it < kIters; ++it) orow[row0 + 4 * it] = __float2bfloat16(outv[it]);
  }
}

}  // namespace gdn
