// GDN decode against a state pool, for T >= 1 tokens per sequence: the
// serving-side forms of the decode step.
//
//   * T = 1 with a pool: each batch entry reads its state from slot
//     read_idx[b] of a [P, H_v, V, K] pool and writes the new state to slot
//     write_idx[b] (= read_idx[b] when no write indices are given), so a serving
//     loop needs no gather/scatter of states around the step.  Semantics follow
//     FlashInfer's gated_delta_rule_decode_pretranspose with initial_state /
//     initial_state_indices / output_state_indices
//     (site flashinfer/gdn_decode.py:117-200).
//   * T > 1 (multi-token prediction / speculative verify): the T tokens of a
//     sequence run in order on the state held in registers, each token's output
//     is written, and optionally the state after every token is kept for
//     rollback in intermediate[read_idx[b], t] (site
//     flashinfer/trace/templates/gdn.py:378-466, _gdn_mtp_reference).
//   * fp32 or bf16 state.  The recurrence runs in fp32 registers either way; a
//     bf16 pool is rounded once per stored state (final and intermediate).
//   * A negative index marks a padding entry: its outputs are written as zero
//     and no state is read or written (the fp32 behaviour of
//     site flashinfer/gdn_decode.py:182-195).  An index >= pool_size is treated
//     the same way and raises GDN_B200_STATUS_BAD_INDEX.
//
// Per token the step is the reference decode step (ref solution/cuda/kernel.cu:21-97):
//   s = g S_v;  delta_v = beta (v_v - <s,k>);  S_v' = s + delta_v k;
//   o_v = scale (<s,q> + delta_v <k,q>)
// with the same thread layout as gdn_decode_kernel: a CTA of 4 warps covers 16
// rows of one (batch, v-head) state, 8 lanes per 512-byte (fp32) or 256-byte
// (bf16) row.
#pragma once

#include "decode_kernel.cuh"

namespace gdn {

constexpr unsigned int kStatusBadIndex = 8u;   // a state index >= pool_size

struct PoolDecodeParams {
  const __nv_bfloat16* q;        // [B, T, H_qk, K]
  const __nv_bfloat16* k;        // [B, T, H_qk, K]
  const __nv_bfloat16* v;        // [B, T, H_v, V]
  const void* pool;              // [P, H_v, V, K] fp32 or bf16
  void* new_pool;                // [P, H_v, V, K], may alias pool
  void* inter;                   // [P, T, H_v, V, K] or nullptr
  const void* read_idx;          // [B] int32 / int64
  const void* write_idx;         // [B] int32 / int64, or nullptr (= read_idx)
  int idx_is_int64;
  const float* A_log;            // [H_v]
  const __nv_bfloat16* a;        // [B, T, H_v]
  const float* dt_bias;          // [H_v]
  const __nv_bfloat16* b;        // [B, T, H_v]
  float scale;
  __nv_bfloat16* out;            // [B, T, H_v, V]
  unsigned int* status;
  long long pool_size;
  int T;
  int h_qk;
  int h_v;
};

__device__ __forceinline__ long long pool_index(const void* idx, int is64, int b) {
  return is64 ? reinterpret_cast<const long long*>(idx)[b]
              : static_cast<long long>(reinterpret_cast<const int*>(idx)[b]);
}

// Four consecutive state elements <-> float4, for either state type.
__device__ __forceinline__ float4 ld_state4(const float* p) { return ld_state(p); }
__device__ __forceinline__ float4 ld_state4(const __nv_bfloat16* p) {
  uint32_t lo, hi;
  asm volatile("ld.global.L1::no_allocate.L2::256B.v2.b32 {%0,%1}, [%2];"
               : "=r"(lo), "=r"(hi)
               : "l"(p));
  const float2 f0 = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&lo));
  const float2 f1 = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&hi));
  return make_float4(f0.x, f0.y, f1.x, f1.y);
}
__device__ __forceinline__ void st_state4(float* p, float4 r) { st_state(p, r); }
__device__ __forceinline__ void st_state4(__nv_bfloat16* p, float4 r) {
  const uint32_t lo = pack_bf16x2(r.x, r.y), hi = pack_bf16x2(r.z, r.w);
  asm volatile("st.global.v2.b32 [%0], {%1,%2};" ::"l"(p), "r"(lo), "r"(hi) : "memory");
}

template <typename StateT>
__global__ void __launch_bounds__(kDecodeThreads) gdn_decode_pool_kernel(PoolDecodeParams p) {
  constexpr int kRows = 16;   // rows per CTA: 4 warps x 4 rows
  constexpr int kCtasPerHead = kHeadDim / kRows;
  const int bh = blockIdx.x / kCtasPerHead;   // batch * H_v + v-head
  const int rblk = blockIdx.x % kCtasPerHead;
  const int h = bh % p.h_v;
  const int bidx = bh / p.h_v;
  const int hq = h / (p.h_v / p.h_qk);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int l8 = lane & 7;
  const int row = rblk * kRows + warp * 4 + (lane >> 3);
  const size_t hd2 = static_cast<size_t>(kHeadDim) * kHeadDim;

  long long ridx = pool_index(p.read_idx, p.idx_is_int64, bidx);
  long long widx = p.write_idx ? pool_index(p.write_idx, p.idx_is_int64, bidx) : ridx;
  if (ridx >= p.pool_size || widx >= p.pool_size) {
    if (threadIdx.x == 0 && rblk == 0) atomicOr(p.status, kStatusBadIndex);
    ridx = -1;
  }
  if (ridx < 0 || widx < 0) {   // padding entry: zero outputs, no state traffic
    if (l8 == 0)
      for (int t = 0; t < p.T; ++t)
        p.out[((static_cast<size_t>(bidx) * p.T + t) * p.h_v + h) * kHeadDim + row] =
            __float2bfloat16(0.f);
    return;
  }

  // This lane's 16 state elements: columns 4*l8 + 32*j + e of row `row`.
  const StateT* src = static_cast<const StateT*>(p.pool) + (ridx * p.h_v + h) * hd2 +
                      static_cast<size_t>(row) * kHeadDim + 4 * l8;
  float4 st[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) st[j] = ld_state4(src + 32 * j);

  const float neg_exp_alog = -expf(p.A_log[h]);
  const float dtb = p.dt_bias[h];
  for (int t = 0; t < p.T; ++t) {
    const size_t tok = static_cast<size_t>(bidx) * p.T + t;
    const size_t gate_off = tok * p.h_v + h;
    const float g = expf(neg_exp_alog * softplus20(__bfloat162float(p.a[gate_off]) + dtb));
    const float beta = 1.0f / (1.0f + expf(-__bfloat162float(p.b[gate_off])));
    const size_t qk_off = (tok * p.h_qk + hq) * kHeadDim;
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

    float s[16];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      s[4 * j + 0] = g * st[j].x; s[4 * j + 1] = g * st[j].y;
      s[4 * j + 2] = g * st[j].z; s[4 * j + 3] = g * st[j].w;
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
    const float vv = __bfloat162float(p.v[(tok * p.h_v + h) * kHeadDim + row]);
    const float delta = beta * (vv - dk);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      st[j].x = fmaf(delta, kf[4 * j + 0], s[4 * j + 0]);
      st[j].y = fmaf(delta, kf[4 * j + 1], s[4 * j + 1]);
      st[j].z = fmaf(delta, kf[4 * j + 2], s[4 * j + 2]);
      st[j].w = fmaf(delta, kf[4 * j + 3], s[4 * j + 3]);
    }
    if (l8 == 0) p.out[(tok * p.h_v + h) * kHeadDim + row] = __float2bfloat16(p.scale * (dq + delta * qk));
    if (p.inter) {   // state after token t, at [read slot, t]
      StateT* dst = static_cast<StateT*>(p.inter) +
                    ((ridx * p.T + t) * p.h_v + h) * hd2 + static_cast<size_t>(row) * kHeadDim +
                    4 * l8;
#pragma unroll
      for (int j = 0; j < 4; ++j) st_state4(dst + 32 * j, st[j]);
    }
  }
  StateT* dst = static_cast<StateT*>(p.new_pool) + (widx * p.h_v + h) * hd2 +
                static_cast<size_t>(row) * kHeadDim + 4 * l8;
#pragma unroll
  for (int j = 0; j < 4; ++j) st_state4(dst + 32 * j, st[j]);
}

}  // namespace gdn
