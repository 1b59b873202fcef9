// GDN decode: one fused, bandwidth-bound pass over the k-last state
// [*, H_v, V, K] per call, for T >= 1 tokens per sequence.
//
// Per token the step is the reference decode step (ref solution/cuda/kernel.cu:21-97):
//   g = exp(-exp(A_log) softplus(a + dt_bias)),  beta = sigmoid(b)
//   S <- g S;  delta = beta (v - S k);  S += delta k^T;  o = scale S q
// written per state row v (rows are independent in the k-last layout):
//   s = g S_v;  delta_v = beta (v_v - <s,k>);  S_v' = s + delta_v k;
//   o_v = scale (<s,q> + delta_v <k,q>)
//
// One kernel serves the reference's decode entry point and its serving forms:
//   * the reference decode (gdn_b200_decode): T = 1, state [B, H_v, V, K] fp32
//     indexed by the batch entry, state == nullptr meaning a zero state
//     (ref kernel.cu:135-139), new_state possibly aliasing state;
//   * a state pool [P, H_v, V, K] (fp32 or bf16): entry b reads slot
//     read_idx[b] and writes slot write_idx[b] (= read_idx[b] when no write
//     indices are given), as FlashInfer's pooled decode
//     (site flashinfer/gdn_decode.py:117-200);
//   * T > 1 tokens per sequence (multi-token prediction / speculative verify):
//     the T tokens run in order on the state held in registers, each token's
//     output is written, and optionally the state after every token is kept in
//     intermediate[read_idx[b], t] (site flashinfer/trace/templates/gdn.py:
//     378-466, _gdn_mtp_reference).
// The recurrence runs in fp32 registers; a bf16 pool is rounded once per stored
// state.  A negative index marks a padding entry: its outputs are written as zero
// and no state is read or written (the fp32 behaviour of site
// flashinfer/gdn_decode.py:182-195).  An index >= pool_size is treated the same
// way and raises kStatusBadIndex.
//
// Layout on the SM: a CTA of 4 warps; eight lanes share one state row, each
// lane owning 16 columns read as 16-byte vectors, so one warp instruction moves
// four rows fully coalesced and the row reductions are 3-level xor shuffles.
// Each thread carries kRowIters rows (two 512-byte fp32 rows, or four 256-byte
// bf16 rows) whose loads are all issued before any use, keeping 16 KiB (fp32)
// or 16 KiB (bf16) of state in flight per CTA.
#pragma once

#include "gdn_ptx.cuh"

namespace gdn {

constexpr int kHeadDim = 128;
constexpr int kDecodeThreads = 128;

__device__ __forceinline__ float softplus20(float x) {
  return x > 20.0f ? x : log1pf(expf(x));
}

// State loads bypass L1 (each byte is read once) and ask L2 for 256-byte
// sectors, the row pair a warp instruction touches.
__device__ __forceinline__ float4 ld_state(const float* p) {
  float4 r;
  asm volatile("ld.global.L1::no_allocate.L2::256B.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ void st_state(float* p, float4 r) {
  asm volatile("st.global.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(p), "f"(r.x), "f"(r.y), "f"(r.z),
               "f"(r.w)
               : "memory");
}

constexpr unsigned int kStatusBadIndex = 8u;   // a state index >= pool_size

struct DecodeParams {
  const __nv_bfloat16* q;        // [B, T, H_qk, K]
  const __nv_bfloat16* k;        // [B, T, H_qk, K]
  const __nv_bfloat16* v;        // [B, T, H_v, V]
  const void* pool;              // [P, H_v, V, K] fp32 or bf16, or nullptr (zero state)
  void* new_pool;                // [P, H_v, V, K], may alias pool
  void* inter;                   // [P, T, H_v, V, K] or nullptr
  const void* read_idx;          // [B] int32 / int64, or nullptr (slot = batch entry)
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

// Per state type: each lane owns 16 columns of a row, read as kAcc vector
// accesses of kVec elements at columns kVec*l8 + 8*kVec*j + e (j < kAcc, e <
// kVec), so every access is 16 bytes and 8 lanes cover a row.  A bf16 row is
// half the bytes, so a bf16 thread carries twice the rows.
template <typename StateT> struct DecodeLayout;
template <> struct DecodeLayout<float> {
  static constexpr int kVec = 4, kAcc = 4, kRowIters = 2;
};
template <> struct DecodeLayout<__nv_bfloat16> {
  static constexpr int kVec = 8, kAcc = 2, kRowIters = 4;
};

__device__ __forceinline__ void ld_vec(const float* p, float* x) {
  const float4 r = ld_state(p);
  x[0] = r.x; x[1] = r.y; x[2] = r.z; x[3] = r.w;
}
__device__ __forceinline__ void ld_vec(const __nv_bfloat16* p, float* x) {
  uint32_t w[4];
  asm volatile("ld.global.L1::no_allocate.L2::256B.v4.b32 {%0,%1,%2,%3}, [%4];"
               : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3])
               : "l"(p));
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&w[i]));
    x[2 * i] = f.x;
    x[2 * i + 1] = f.y;
  }
}
__device__ __forceinline__ void st_vec(float* p, const float* x) {
  st_state(p, make_float4(x[0], x[1], x[2], x[3]));
}
__device__ __forceinline__ void st_vec(__nv_bfloat16* p, const float* x) {
  asm volatile("st.global.v4.b32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(pack_bf16x2(x[0], x[1])),
               "r"(pack_bf16x2(x[2], x[3])), "r"(pack_bf16x2(x[4], x[5])),
               "r"(pack_bf16x2(x[6], x[7]))
               : "memory");
}

// One token's inputs for this thread, kept as packed bf16 until used: the q/k
// fragments (16 columns each), the gate inputs and this thread's v entries.
template <int kRowIters>
struct TokIn {
  uint32_t q[8], k[8];
  __nv_bfloat16 a, b, v[kRowIters];
};

// kVec consecutive bf16 (kVec / 2 words) from global memory.
template <int kVec>
__device__ __forceinline__ void ld_words(const __nv_bfloat16* p, uint32_t* w) {
  if constexpr (kVec == 4) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    w[0] = u.x; w[1] = u.y;
  } else {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    w[0] = u.x; w[1] = u.y; w[2] = u.z; w[3] = u.w;
  }
}

__device__ __forceinline__ void unpack16(const uint32_t* w, float* x) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
    x[2 * i] = f.x;
    x[2 * i + 1] = f.y;
  }
}

// 16-byte global -> shared copies that bypass registers (both addresses
// 16-byte aligned), committed as one group and waited for together.
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gsrc)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_all;" ::: "memory");
}
// All but the most recently committed group have landed.
__device__ __forceinline__ void cp_async_wait_group1() {
  asm volatile("cp.async.wait_group 1;" ::: "memory");
}

// kVec state elements from shared memory as floats (the layout of ld_vec).
__device__ __forceinline__ void ld_vec_smem(const float* p, float* x) {
  const float4 r = *reinterpret_cast<const float4*>(p);
  x[0] = r.x; x[1] = r.y; x[2] = r.z; x[3] = r.w;
}
__device__ __forceinline__ void ld_vec_smem(const __nv_bfloat16* p, float* x) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
    x[2 * i] = f.x;
    x[2 * i + 1] = f.y;
  }
}

// Tokens whose inputs a CTA stages in shared memory at a time (T > 1).
constexpr int kTokGroup = 16;

// kHasState = false is the reference decode's null state (a zero initial state,
// no state reads).  kMulti = false is the T = 1 instance: the token's inputs go
// straight to registers.  kMulti = true stages the inputs of up to kTokGroup tokens in
// shared memory with one round of loads, so the per-token steps do not each
// wait out a global-memory latency.
// The bf16-pool one-token instance is held to 6 CTAs per SM (80 registers, a
// few spilled): with its state packed that keeps more state bytes in flight
// per SM than 4 spill-free CTAs do (27.7 against 30.6 us at B=64 on B200).
template <typename StateT, bool kMulti, bool kHasState>
__global__ void __launch_bounds__(kDecodeThreads, (!kMulti && sizeof(StateT) == 2) ? 6 : 0)
    gdn_decode_kernel(DecodeParams p) {
  using L = DecodeLayout<StateT>;
  constexpr int kVec = L::kVec, kAcc = L::kAcc, kRI = L::kRowIters;
  constexpr int kRows = 16 * kRI;   // rows per CTA: 4 warps x 4 rows x kRowIters
  constexpr int kCtasPerHead = kHeadDim / kRows;
  // Multi-token calls of up to kTokGroup tokens give each CTA two consecutive
  // row blocks (2 x kRows rows of one head): the second block's state streams
  // into shared memory while the first block's tokens run.
  const bool pair = kMulti && p.T <= kTokGroup;
  const int per_head = pair ? kCtasPerHead / 2 : kCtasPerHead;
  const int bh = blockIdx.x / per_head;   // batch * H_v + v-head
  const int rblk = (blockIdx.x % per_head) * (pair ? 2 : 1);
  const int h = bh % p.h_v;
  const int bidx = bh / p.h_v;
  const int hq = h / (p.h_v / p.h_qk);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int l8 = lane & 7;
  int row0 = rblk * kRows + warp * (4 * kRI) + (lane >> 3);   // rows row0 + 4 i (this block)
  const size_t hd2 = static_cast<size_t>(kHeadDim) * kHeadDim;

  // Token inputs of token t (issued before they are needed: the slot index
  // load, then token 0's inputs, then the state rows).
  auto load_tok = [&](int t, TokIn<kRI>& in) {
    const size_t tok = static_cast<size_t>(bidx) * p.T + t;
    const size_t qk_off = (tok * p.h_qk + hq) * kHeadDim;
#pragma unroll
    for (int j = 0; j < kAcc; ++j) {
      ld_words<kVec>(p.q + qk_off + kVec * l8 + 8 * kVec * j, in.q + (kVec / 2) * j);
      ld_words<kVec>(p.k + qk_off + kVec * l8 + 8 * kVec * j, in.k + (kVec / 2) * j);
    }
    in.a = p.a[tok * p.h_v + h];
    in.b = p.b[tok * p.h_v + h];
#pragma unroll
    for (int i = 0; i < kRI; ++i) in.v[i] = p.v[(tok * p.h_v + h) * kHeadDim + row0 + 4 * i];
  };

  // Slots: the batch entry itself without indices (the reference decode).
  long long ridx = p.read_idx ? pool_index(p.read_idx, p.idx_is_int64, bidx) : bidx;
  long long widx = p.write_idx ? pool_index(p.write_idx, p.idx_is_int64, bidx) : ridx;
  TokIn<kRI> cur;
  if constexpr (!kMulti) load_tok(0, cur);
  if (ridx >= p.pool_size || widx >= p.pool_size) {
    if (threadIdx.x == 0 && rblk == 0) atomicOr(p.status, kStatusBadIndex);
    ridx = -1;
  }
  if (ridx < 0 || widx < 0) {   // padding entry: zero outputs, no state traffic
    if (l8 == 0)
      for (int t = 0; t < p.T; ++t)
        for (int blk = 0; blk < (pair ? 2 : 1); ++blk)
#pragma unroll
          for (int i = 0; i < kRI; ++i)
            p.out[((static_cast<size_t>(bidx) * p.T + t) * p.h_v + h) * kHeadDim + row0 +
                  blk * kRows + 4 * i] = __float2bfloat16(0.f);
    return;
  }

  if constexpr (sizeof(StateT) == 2 && !kMulti && kHasState) {
    // bf16 pool, one token.  The state rows stay packed, two bf16 per 32-bit
    // register (32 registers instead of 64 floats), and are unpacked row by
    // row: fewer registers per thread, more CTAs and so more state bytes in
    // flight per SM.  The arithmetic and its order are those of the general
    // path below, so the results are the same bits.
    const size_t base = (ridx * p.h_v + h) * hd2 + static_cast<size_t>(row0) * kHeadDim + kVec * l8;
    const __nv_bfloat16* srcb = static_cast<const __nv_bfloat16*>(p.pool) + base;
    uint32_t raw[kRI][8];
#pragma unroll
    for (int i = 0; i < kRI; ++i)
#pragma unroll
      for (int j = 0; j < 2; ++j)
        asm volatile("ld.global.L1::no_allocate.L2::256B.v4.b32 {%0,%1,%2,%3}, [%4];"
                     : "=r"(raw[i][4 * j]), "=r"(raw[i][4 * j + 1]), "=r"(raw[i][4 * j + 2]),
                       "=r"(raw[i][4 * j + 3])
                     : "l"(srcb + 4 * i * kHeadDim + 8 * kVec * j));
    auto unpack2 = [](uint32_t w) {
      return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w));
    };
    const float g = expf(-expf(p.A_log[h]) * softplus20(__bfloat162float(cur.a) + p.dt_bias[h]));
    const float beta = 1.0f / (1.0f + expf(-__bfloat162float(cur.b)));
    float qk = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      const float2 q2 = unpack2(cur.q[w]), k2 = unpack2(cur.k[w]);
      qk = fmaf(q2.x, k2.x, qk);
      qk = fmaf(q2.y, k2.y, qk);
    }
    qk += __shfl_xor_sync(0xffffffffu, qk, 1);
    qk += __shfl_xor_sync(0xffffffffu, qk, 2);
    qk += __shfl_xor_sync(0xffffffffu, qk, 4);
#pragma unroll
    for (int i = 0; i < kRI; ++i) {
      float dk = 0.f, dq = 0.f;
#pragma unroll
      for (int w = 0; w < 8; ++w) {
        const float2 s2 = unpack2(raw[i][w]), k2 = unpack2(cur.k[w]), q2 = unpack2(cur.q[w]);
        const float sx = g * s2.x, sy = g * s2.y;
        dk = fmaf(sx, k2.x, dk);
        dq = fmaf(sx, q2.x, dq);
        dk = fmaf(sy, k2.y, dk);
        dq = fmaf(sy, q2.y, dq);
      }
#pragma unroll
      for (int m = 1; m < 8; m <<= 1) {
        dk += __shfl_xor_sync(0xffffffffu, dk, m);
        dq += __shfl_xor_sync(0xffffffffu, dq, m);
      }
      const float delta = beta * (__bfloat162float(cur.v[i]) - dk);
#pragma unroll
      for (int w = 0; w < 8; ++w) {
        const float2 s2 = unpack2(raw[i][w]), k2 = unpack2(cur.k[w]);
        raw[i][w] = pack_bf16x2(fmaf(delta, k2.x, g * s2.x), fmaf(delta, k2.y, g * s2.y));
      }
      if (l8 == 0)
        p.out[(static_cast<size_t>(bidx) * p.h_v + h) * kHeadDim + row0 + 4 * i] =
            __float2bfloat16(p.scale * (dq + delta * qk));
    }
    auto store_rows = [&](__nv_bfloat16* dst) {
#pragma unroll
      for (int i = 0; i < kRI; ++i)
#pragma unroll
        for (int j = 0; j < 2; ++j)
          asm volatile("st.global.v4.b32 [%0], {%1,%2,%3,%4};" ::"l"(
                           dst + 4 * i * kHeadDim + 8 * kVec * j),
                       "r"(raw[i][4 * j]), "r"(raw[i][4 * j + 1]), "r"(raw[i][4 * j + 2]),
                       "r"(raw[i][4 * j + 3])
                       : "memory");
    };
    if (p.inter)   // the state after the token, at [read slot, 0]
      store_rows(static_cast<__nv_bfloat16*>(p.inter) + base);
    store_rows(static_cast<__nv_bfloat16*>(p.new_pool) + (widx * p.h_v + h) * hd2 +
               static_cast<size_t>(row0) * kHeadDim + kVec * l8);
    return;
  }

  // This thread's state: rows row0 + 4 i, 16 columns each.
  const StateT* src = static_cast<const StateT*>(p.pool) + (ridx * p.h_v + h) * hd2 +
                      static_cast<size_t>(row0) * kHeadDim + kVec * l8;
  float st[kRI][16];
  if constexpr (kHasState) {
#pragma unroll
    for (int i = 0; i < kRI; ++i)
#pragma unroll
      for (int j = 0; j < kAcc; ++j)
        ld_vec(src + 4 * i * kHeadDim + 8 * kVec * j, st[i] + kVec * j);
  } else {   // no state: a zero initial state (ref kernel.cu:135-139)
#pragma unroll
    for (int i = 0; i < kRI; ++i)
#pragma unroll
      for (int e = 0; e < 16; ++e) st[i][e] = 0.f;
  }

  const float neg_exp_alog = -expf(p.A_log[h]);
  const float dtb = p.dt_bias[h];
  // Gate and beta of one token (ref kernel.cu:44-53).
  auto gates = [&](float av, float bv, float& g, float& beta) {
    g = expf(neg_exp_alog * softplus20(av + dtb));
    beta = 1.0f / (1.0f + expf(-bv));
  };
  // One token step on this thread's rows (inputs already unpacked, gates formed).
  // (The multi-token instance passes q.k in, formed once per staged token.)
  auto step = [&](int t, const float* qf, const float* kf, float g, float beta,
                  const float* vv, float qk_pre) {
    const size_t tok = static_cast<size_t>(bidx) * p.T + t;
    float qk = qk_pre;
    if constexpr (!kMulti) {
      qk = 0.f;
#pragma unroll
      for (int e = 0; e < 16; ++e) qk = fmaf(qf[e], kf[e], qk);
      qk += __shfl_xor_sync(0xffffffffu, qk, 1);
      qk += __shfl_xor_sync(0xffffffffu, qk, 2);
      qk += __shfl_xor_sync(0xffffffffu, qk, 4);
    }
#pragma unroll
    for (int i = 0; i < kRI; ++i) {
      if constexpr (kMulti) {
        // Several tokens run back to back on the state in registers, so this
        // product is on the path from one token to the next: four short
        // chains instead of one of 16.  The steps are issue-bound, so the
        // element-wise work runs as packed pairs (sm_100 f32x2 multiply and
        // fma, each lane rounded exactly as the scalar instruction): the
        // decay, the chains (accumulators 0-1 and 2-3 as pairs) and the update.
        const float2 g2 = make_float2(g, g);
        float2 s2[8];
#pragma unroll
        for (int m = 0; m < 8; ++m)
          s2[m] = __fmul2_rn(g2, make_float2(st[i][2 * m], st[i][2 * m + 1]));
        float2 ak01 = make_float2(0.f, 0.f), ak23 = ak01, aq01 = ak01, aq23 = ak01;
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          const int e = 4 * m;
          ak01 = __ffma2_rn(s2[2 * m], make_float2(kf[e], kf[e + 1]), ak01);
          ak23 = __ffma2_rn(s2[2 * m + 1], make_float2(kf[e + 2], kf[e + 3]), ak23);
          aq01 = __ffma2_rn(s2[2 * m], make_float2(qf[e], qf[e + 1]), aq01);
          aq23 = __ffma2_rn(s2[2 * m + 1], make_float2(qf[e + 2], qf[e + 3]), aq23);
        }
        float dk = (ak01.x + ak01.y) + (ak23.x + ak23.y);
        float dq = (aq01.x + aq01.y) + (aq23.x + aq23.y);
#pragma unroll
        for (int m = 1; m < 8; m <<= 1) {
          dk += __shfl_xor_sync(0xffffffffu, dk, m);
          dq += __shfl_xor_sync(0xffffffffu, dq, m);
        }
        const float delta = beta * (vv[i] - dk);
        const float2 d2 = make_float2(delta, delta);
#pragma unroll
        for (int m = 0; m < 8; ++m) {
          const float2 u = __ffma2_rn(d2, make_float2(kf[2 * m], kf[2 * m + 1]), s2[m]);
          st[i][2 * m] = u.x;
          st[i][2 * m + 1] = u.y;
        }
        if (l8 == 0)
          p.out[(tok * p.h_v + h) * kHeadDim + row0 + 4 * i] =
              __float2bfloat16(p.scale * (dq + delta * qk));
      } else {
        float s[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) s[e] = g * st[i][e];
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
        const float delta = beta * (vv[i] - dk);
#pragma unroll
        for (int e = 0; e < 16; ++e) st[i][e] = fmaf(delta, kf[e], s[e]);
        if (l8 == 0)
          p.out[(tok * p.h_v + h) * kHeadDim + row0 + 4 * i] =
              __float2bfloat16(p.scale * (dq + delta * qk));
      }
    }
    if (p.inter) {   // state after token t, at [read slot, t]
      StateT* dst = static_cast<StateT*>(p.inter) + ((ridx * p.T + t) * p.h_v + h) * hd2 +
                    static_cast<size_t>(row0) * kHeadDim + kVec * l8;
#pragma unroll
      for (int i = 0; i < kRI; ++i)
#pragma unroll
        for (int j = 0; j < kAcc; ++j)
          st_vec(dst + 4 * i * kHeadDim + 8 * kVec * j, st[i] + kVec * j);
    }
  };

  if constexpr (!kMulti) {
    float qf[16], kf[16], vv[kRI];
    unpack16(cur.q, qf);
    unpack16(cur.k, kf);
#pragma unroll
    for (int i = 0; i < kRI; ++i) vv[i] = __bfloat162float(cur.v[i]);
    float g, beta;
    gates(__bfloat162float(cur.a), __bfloat162float(cur.b), g, beta);
    step(0, qf, kf, g, beta, vv, 0.f);
  } else {
    // Staged token inputs: q and k rows (256 B each), a, b, and this CTA's v rows.
    __shared__ __align__(16) __nv_bfloat16 sq[kTokGroup][kHeadDim];
    __shared__ __align__(16) __nv_bfloat16 sk[kTokGroup][kHeadDim];
    __shared__ float sa[kTokGroup], sb[kTokGroup];
    __shared__ __align__(16) __nv_bfloat16 sv[kTokGroup][2 * kRows];
    __shared__ __align__(16) StateT sst[kRows][kHeadDim];   // the second row block's state
    // q.k of each staged token, per warp (written and read by the same warp).
    __shared__ float sqk[kDecodeThreads / 32][kTokGroup];
    const int tid = threadIdx.x;
    const int vrows = pair ? 2 * kRows : kRows;
    // This lane's 16 columns of staged token tt's q and k, as floats.
    auto load_qk = [&](int tt, float* qf, float* kf) {
#pragma unroll
      for (int j = 0; j < kAcc; ++j) {
        uint32_t wq[kVec / 2], wk[kVec / 2];
        if constexpr (kVec == 4) {
          const uint2 uq = *reinterpret_cast<const uint2*>(&sq[tt][kVec * l8 + 8 * kVec * j]);
          const uint2 uk = *reinterpret_cast<const uint2*>(&sk[tt][kVec * l8 + 8 * kVec * j]);
          wq[0] = uq.x; wq[1] = uq.y; wk[0] = uk.x; wk[1] = uk.y;
        } else {
          const uint4 uq = *reinterpret_cast<const uint4*>(&sq[tt][kVec * l8 + 8 * kVec * j]);
          const uint4 uk = *reinterpret_cast<const uint4*>(&sk[tt][kVec * l8 + 8 * kVec * j]);
          wq[0] = uq.x; wq[1] = uq.y; wq[2] = uq.z; wq[3] = uq.w;
          wk[0] = uk.x; wk[1] = uk.y; wk[2] = uk.z; wk[3] = uk.w;
        }
#pragma unroll
        for (int w = 0; w < kVec / 2; ++w) {
          const float2 fq = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&wq[w]));
          const float2 fk = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&wk[w]));
          qf[kVec * j + 2 * w] = fq.x; qf[kVec * j + 2 * w + 1] = fq.y;
          kf[kVec * j + 2 * w] = fk.x; kf[kVec * j + 2 * w + 1] = fk.y;
        }
      }
    };
    // One staged token group's steps on this thread's rows.
    auto run_tokens = [&](int t0, int n) {
        for (int tt = 0; tt < n; ++tt) {
          float qf[16], kf[16], vv[kRI];
          load_qk(tt, qf, kf);
#pragma unroll
          for (int i = 0; i < kRI; ++i)
            vv[i] = __bfloat162float(sv[tt][row0 - rblk * kRows + 4 * i]);
          step(t0 + tt, qf, kf, sa[tt], sb[tt], vv, sqk[warp][tt]);
        }
    };
    for (int t0 = 0; t0 < p.T; t0 += kTokGroup) {
      const int n = min(kTokGroup, p.T - t0);
      __syncthreads();   // the previous group is consumed
      // The group's q/k rows and this CTA's v entries go straight from global
      // to shared memory (cp.async, no registers held), all in flight
      // together: one memory latency per group, which on the first group
      // overlaps the state rows'.
      for (int e = tid; e < n * 16; e += kDecodeThreads) {   // 16 x 16 B per q/k row
        const int tt = e >> 4, c = e & 15;
        const size_t qk_off =
            ((static_cast<size_t>(bidx) * p.T + t0 + tt) * p.h_qk + hq) * kHeadDim + 8 * c;
        cp_async16(&sq[tt][8 * c], p.q + qk_off);
        cp_async16(&sk[tt][8 * c], p.k + qk_off);
      }
      for (int e = tid; e < n * (vrows / 8); e += kDecodeThreads) {   // 16 B of v rows
        const int tt = e / (vrows / 8), c = e % (vrows / 8);
        cp_async16(&sv[tt][8 * c],
                   p.v + ((static_cast<size_t>(bidx) * p.T + t0 + tt) * p.h_v + h) * kHeadDim +
                       rblk * kRows + 8 * c);
      }
      cp_async_commit();
      if (pair) {   // the second block's state rows, a later group: still in flight below
        constexpr int kChunksPerRow = kHeadDim * static_cast<int>(sizeof(StateT)) / 16;
        const StateT* src2 = static_cast<const StateT*>(p.pool) + (ridx * p.h_v + h) * hd2 +
                             static_cast<size_t>(rblk + 1) * kRows * kHeadDim;
        for (int e = tid; e < kRows * kChunksPerRow; e += kDecodeThreads) {
          const int r = e / kChunksPerRow, c = e % kChunksPerRow;
          cp_async16(reinterpret_cast<uint8_t*>(&sst[r][0]) + 16 * c,
                     reinterpret_cast<const uint8_t*>(src2 + static_cast<size_t>(r) * kHeadDim) +
                         16 * c);
        }
        cp_async_commit();
      }
      float ga = 0.f, gb = 0.f;
      if (tid < n) {
        const size_t gate_off = (static_cast<size_t>(bidx) * p.T + t0 + tid) * p.h_v + h;
        ga = __bfloat162float(p.a[gate_off]);
        gb = __bfloat162float(p.b[gate_off]);
      }
      if (pair) cp_async_wait_group1();   // the token group has landed
      else cp_async_wait_all();
      // the group's gates, formed once for all rows (sa = g, sb = beta)
      if (tid < n) gates(ga, gb, sa[tid], sb[tid]);
      __syncthreads();
      // q.k of the group's tokens once per warp, not once per token step and
      // row block: four tokens per pass, eight lanes each, over the columns
      // and the xor tree a token step uses, so the sums are the same bits.
      for (int p0 = 0; p0 < n; p0 += 4) {
        const int tt = p0 + (lane >> 3);
        float part = 0.f;
        if (tt < n) {
          float qf[16], kf[16];
          load_qk(tt, qf, kf);
#pragma unroll
          for (int e = 0; e < 16; ++e) part = fmaf(qf[e], kf[e], part);
        }
        part += __shfl_xor_sync(0xffffffffu, part, 1);
        part += __shfl_xor_sync(0xffffffffu, part, 2);
        part += __shfl_xor_sync(0xffffffffu, part, 4);
        if (tt < n && l8 == 0) sqk[warp][tt] = part;
      }
      __syncwarp();
      run_tokens(t0, n);
    }
    if (pair) {
      // First block done: its state out, then the second block's from shared
      // memory, and the same staged tokens (one group: T <= kTokGroup) again.
      StateT* dst1 = static_cast<StateT*>(p.new_pool) + (widx * p.h_v + h) * hd2 +
                     static_cast<size_t>(row0) * kHeadDim + kVec * l8;
#pragma unroll
      for (int i = 0; i < kRI; ++i)
#pragma unroll
        for (int j = 0; j < kAcc; ++j)
          st_vec(dst1 + 4 * i * kHeadDim + 8 * kVec * j, st[i] + kVec * j);
      cp_async_wait_all();
      __syncthreads();
      row0 += kRows;
#pragma unroll
      for (int i = 0; i < kRI; ++i)
#pragma unroll
        for (int j = 0; j < kAcc; ++j)
          ld_vec_smem(&sst[row0 - (rblk + 1) * kRows + 4 * i][kVec * l8 + 8 * kVec * j],
                      st[i] + kVec * j);
      run_tokens(0, p.T);
    }
  }
  StateT* dst = static_cast<StateT*>(p.new_pool) + (widx * p.h_v + h) * hd2 +
                static_cast<size_t>(row0) * kHeadDim + kVec * l8;
#pragma unroll
  for (int i = 0; i < kRI; ++i)
#pragma unroll
    for (int j = 0; j < kAcc; ++j) st_vec(dst + 4 * i * kHeadDim + 8 * kVec * j, st[i] + kVec * j);
}

// CTAs per (batch, v-head) of gdn_decode_kernel<StateT, *>.
template <typename StateT>
constexpr int decode_ctas_per_head() {
  return kHeadDim / (16 * DecodeLayout<StateT>::kRowIters);
}

// Launch for `batch` entries; the instance follows the state type, T and
// whether there is a state (multi-token and pooled calls always have one).
inline void launch_decode(const DecodeParams& p, long long batch, bool state_bf16,
                          cudaStream_t st) {
  // multi-token calls of up to kTokGroup tokens: two row blocks per CTA
  const long long div = (p.T > 1 && p.T <= kTokGroup) ? 2 : 1;
  if (state_bf16) {
    const dim3 grid(
        static_cast<unsigned>(batch * p.h_v * decode_ctas_per_head<__nv_bfloat16>() / div));
    if (p.T > 1)
      gdn_decode_kernel<__nv_bfloat16, true, true><<<grid, kDecodeThreads, 0, st>>>(p);
    else
      gdn_decode_kernel<__nv_bfloat16, false, true><<<grid, kDecodeThreads, 0, st>>>(p);
  } else {
    const dim3 grid(static_cast<unsigned>(batch * p.h_v * decode_ctas_per_head<float>() / div));
    if (p.T > 1)
      gdn_decode_kernel<float, true, true><<<grid, kDecodeThreads, 0, st>>>(p);
    else if (p.pool)
      gdn_decode_kernel<float, false, true><<<grid, kDecodeThreads, 0, st>>>(p);
    else
      gdn_decode_kernel<float, false, false><<<grid, kDecodeThreads, 0, st>>>(p);
  }
}

}  // namespace gdn
