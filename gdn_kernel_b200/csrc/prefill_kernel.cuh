// GDN chunked prefill (C = 64) over packed variable-length sequences, with the
// chunk-local contractions on tcgen05 tensor cores (bf16 operands in shared
// memory, fp32 accumulators in TMEM) and tiles brought in by TMA.
//
// Semantics follow the reference prefill kernel (ref solution/cuda/kernel_prefill.cu:36-298).
// Per chunk of L <= 64 tokens of one (sequence, v-head), with S the fp32 state
// [V, K] entering the chunk:
//   gamma = inclusive cumsum of log g;  beta = sigmoid(b)               (ref :101-122)
//   A_ij  = -beta_i <k_i,k_j> e^{gamma_i-gamma_j}  (i > j)               (ref :134-146)
//   T     = (I - A)^{-1}                                               (ref :148-163)
//   P_ij  = <q_i,k_j> e^{gamma_i-gamma_j}  (j <= i)                      (ref :165-185)
//   W     = T diag(beta e^gamma) K,  U = T diag(beta) V                  (ref :187-195, :248-271)
//   v_new = U - W S^T                                                  (ref :236-271)
//   O     = scale ((e^gamma Q) S^T + P v_new)                          (ref :211-234, :273-284)
//   S     = e^{gamma_last} S + v_new^T (K e^{gamma_last - gamma})      (ref :197-202, :286-293)
//
// B200 mapping.  One CTA (8 warps) per (sequence, v-head) walks its chunks in
// order.  Every UMMA is M = 128 (TMEM lane = matrix row): 64-row operands are
// stacked in shared memory so one instruction stream serves two products:
//   D_QK [128x64]  = [Q ; K] K^T             rows 0-63 Q K^T, rows 64-127 K K^T
//   D_W  [128x128] = [T' ; P] K              rows 0-63 W  (T' = T diag(beta e^gamma))
//   D_UO [128x128] = [Z ; T_b] V             rows 64-127 U (Z is a zero block)
//   D_UO          += [e^g Q ; -W] S^T        rows 0-63 inter, rows 64-127 v_new
//   D_UO          += [P ; Z] v_new           rows 0-63 inter + P v_new
//   D_S4 [128x128] = K^T (v_new e^{gamma_last-gamma})   (S^T increment)
// The fp32 state lives in registers of the 256 threads (thread = TMEM lane k,
// column half), its bf16 copy is the MN-major B operand of the S^T products.
// The 64x64 triangular inverse runs in fp32 on CUDA cores (blocked 16x16).
//
// Every mbarrier wait is bounded; on a timeout the CTA records a status bit,
// stops, frees its TMEM and returns.
#pragma once

#include <cuda.h>
#include "gdn_ptx.cuh"

namespace gdn {

constexpr int kChunk = 64;
constexpr int kPrefillThreads = 256;

// Shared-memory map (byte offsets from a 1024-byte aligned base).
constexpr uint32_t kOffQKW = 0;                    // 32 KiB: K-major [128 rows][128], 2 K-columns of 16 KiB
                                                   //   rows 0-63 Q then e^g Q, rows 64-127 K then -W
constexpr uint32_t kOffKB = kOffQKW + 32768;       // 16 KiB: K chunk [c][kd], kd-blocks of 8 KiB
constexpr uint32_t kOffVB = kOffKB + 16384;        // 16 KiB: V chunk [c][v], v-blocks of 8 KiB
constexpr uint32_t kOffTPZT = kOffVB + 16384;      // 32 KiB: T' | P | Z | T_b, 64x64 bf16 K-major each
constexpr uint32_t kOffSB = kOffTPZT + 32768;      // 32 KiB: S^T bf16 [kd][v], v-blocks of 16 KiB
constexpr uint32_t kOffVN = kOffSB + 32768;        // 16 KiB: v_new [c][v]
constexpr uint32_t kOffVND = kOffVN + 16384;       // 16 KiB: v_new e^{gamma_last-gamma_c}
constexpr int kLdA = 65;                           // fp32 row pitch of A and T
constexpr uint32_t kOffAF = kOffVND + 16384;       // fp32 A [64][65]
constexpr uint32_t kOffTF = kOffAF + 64 * kLdA * 4;  // fp32 T [64][65]
constexpr uint32_t kOffXS = kOffTF + 64 * kLdA * 4;  // fp32 scratch, 3 blocks of 16x16
constexpr uint32_t kOffGam = kOffXS + 3 * 256 * 4;   // gamma[64]
constexpr uint32_t kOffBeta = kOffGam + 256;         // beta[64]
constexpr uint32_t kOffEG = kOffBeta + 256;          // e^gamma[64]
constexpr uint32_t kOffBar = kOffEG + 256;           // 2 mbarriers
constexpr uint32_t kOffTmemPtr = kOffBar + 16;
constexpr uint32_t kSmemUsed = kOffTmemPtr + 16;
constexpr uint32_t kPrefillSmem = kSmemUsed + 1024;  // slack to align the base

// TMEM column map (512 columns allocated, fp32 accumulators, lane = row).
constexpr uint32_t kTmQK = 0;
constexpr uint32_t kTmW = 64;
constexpr uint32_t kTmUO = 192;
constexpr uint32_t kTmS4 = 320;
constexpr uint32_t kTmCols = 512;

constexpr uint32_t kTmaBytesPerChunk = 8 * 8192;   // Q, K (twice), V: 2 boxes each

struct PrefillParams {
  const float* state;            // [N, H_v, V, K] or nullptr (zero state)
  const float* A_log;            // [H_v]
  const __nv_bfloat16* a;        // [T, H_v]
  const float* dt_bias;          // [H_v]
  const __nv_bfloat16* b;        // [T, H_v]
  const void* cu_seqlens;        // [N + 1] int32 or int64
  int cu_is_int64;
  long long total_tokens;
  float scale;
  __nv_bfloat16* out;            // [T, H_v, V]
  float* new_state;              // [N, H_v, V, K], may alias state
  int h_qk;
  int h_v;
  unsigned int* status;          // device status word
};

__device__ __forceinline__ float softplus20p(float x) {
  return x > 20.0f ? x : log1pf(expf(x));
}

__device__ __forceinline__ long long load_cu(const PrefillParams& p, int i) {
  return p.cu_is_int64 ? reinterpret_cast<const long long*>(p.cu_seqlens)[i]
                       : static_cast<long long>(reinterpret_cast<const int*>(p.cu_seqlens)[i]);
}

// Store 64 fp32 values as one 128-byte bf16 row of a 128B-swizzled tile.
__device__ __forceinline__ void st_row_bf16(uint8_t* tile, uint32_t row, const float* x,
                                            float mul) {
#pragma unroll
  for (int cc = 0; cc < 8; ++cc) {
    uint4 u;
    u.x = pack_bf16x2(x[8 * cc + 0] * mul, x[8 * cc + 1] * mul);
    u.y = pack_bf16x2(x[8 * cc + 2] * mul, x[8 * cc + 3] * mul);
    u.z = pack_bf16x2(x[8 * cc + 4] * mul, x[8 * cc + 5] * mul);
    u.w = pack_bf16x2(x[8 * cc + 6] * mul, x[8 * cc + 7] * mul);
    *reinterpret_cast<uint4*>(tile + sw128_off(row, cc)) = u;
  }
}

// Store 32 fp32 values as half (chunks c0..c0+3) of a 128-byte bf16 row.
__device__ __forceinline__ void st_half_row_bf16(uint8_t* tile, uint32_t row, uint32_t c0,
                                                 const float* x, float mul) {
#pragma unroll
  for (int cc = 0; cc < 4; ++cc) {
    uint4 u;
    u.x = pack_bf16x2(x[8 * cc + 0] * mul, x[8 * cc + 1] * mul);
    u.y = pack_bf16x2(x[8 * cc + 2] * mul, x[8 * cc + 3] * mul);
    u.z = pack_bf16x2(x[8 * cc + 4] * mul, x[8 * cc + 5] * mul);
    u.w = pack_bf16x2(x[8 * cc + 6] * mul, x[8 * cc + 7] * mul);
    *reinterpret_cast<uint4*>(tile + sw128_off(row, c0 + cc)) = u;
  }
}

// T = (I - A)^{-1} for the strictly lower 64x64 fp32 A, blocked in 16x16:
//   T_ii = (I - A_ii)^{-1}                  (forward substitution per column)
//   T_ij = T_ii sum_{k=j}^{i-1} A_ik T_kj  (i > j, by block diagonals)
// Only the lower triangle (including the unit diagonal) of T is written.
__device__ __forceinline__ void solve_unit_lower(const float* A, float* T, float* X, int tid) {
  if (tid < 64) {
    const int blk = tid >> 4, j = tid & 15, o = 16 * blk;
    float x[16];
#pragma unroll
    for (int m = 0; m < 16; ++m) {
      float acc = (m == j) ? 1.0f : 0.0f;
#pragma unroll
      for (int l = 0; l < m; ++l) acc = fmaf(A[(o + m) * kLdA + o + l], x[l], acc);
      x[m] = acc;
    }
#pragma unroll
    for (int m = 0; m < 16; ++m) T[(o + m) * kLdA + o + j] = x[m];
  }
  __syncthreads();
#pragma unroll 1
  for (int d = 1; d < 4; ++d) {
    const int nblk = 4 - d;
    // X_i = sum_{k=i-d}^{i-1} A_{i,k} T_{k,i-d}, blocks i = d..3
    for (int e = tid; e < nblk * 256; e += kPrefillThreads) {
      const int i = d + (e >> 8), m = (e >> 4) & 15, n = e & 15, jb = i - d;
      float acc = 0.f;
      for (int kb = jb; kb < i; ++kb) {
#pragma unroll
        for (int l = 0; l < 16; ++l)
          acc = fmaf(A[(16 * i + m) * kLdA + 16 * kb + l], T[(16 * kb + l) * kLdA + 16 * jb + n], acc);
      }
      X[e] = acc;
    }
    __syncthreads();
    // T_{i,i-d} = T_ii X_i
    for (int e = tid; e < nblk * 256; e += kPrefillThreads) {
      const int i = d + (e >> 8), m = (e >> 4) & 15, n = e & 15, jb = i - d;
      const float* Xi = X + (e & ~255);
      float acc = 0.f;
#pragma unroll
      for (int l = 0; l < 16; ++l)
        if (l <= m) acc = fmaf(T[(16 * i + m) * kLdA + 16 * i + l], Xi[l * 16 + n], acc);
      T[(16 * i + m) * kLdA + 16 * jb + n] = acc;
    }
    __syncthreads();
  }
}

__global__ void __launch_bounds__(kPrefillThreads, 1)
    gdn_prefill_kernel(const __grid_constant__ CUtensorMap tm_q,
                       const __grid_constant__ CUtensorMap tm_k,
                       const __grid_constant__ CUtensorMap tm_v, const PrefillParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));

  const int head = blockIdx.x;
  const int seq = blockIdx.y;
  const int hq = head / (p.h_v / p.h_qk);
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int quad = warp & 3;          // TMEM lane quadrant of this warp
  const int half = warp >> 2;         // column half handled by this thread
  const int row = quad * 32 + lane;   // TMEM lane (matrix row) of this thread

  long long s0 = load_cu(p, seq), s1 = load_cu(p, seq + 1);
  if (s0 < 0 || s1 > p.total_tokens || s0 > p.total_tokens) {
    if (tid == 0) atomicOr(p.status, kStatusBadSeqlens);   // treated as an empty sequence
    s1 = s0;
  }
  const long long len = s1 - s0;
  const size_t sbase = (static_cast<size_t>(seq) * p.h_v + head) * kHeadDim * kHeadDim;

  if (len <= 0) {  // ref kernel_prefill.cu:61-66: the state passes through unchanged
    float4* dst = reinterpret_cast<float4*>(p.new_state + sbase);
    const float4* src = p.state ? reinterpret_cast<const float4*>(p.state + sbase) : nullptr;
    for (int i = tid; i < kHeadDim * kHeadDim / 4; i += kPrefillThreads)
      dst[i] = src ? src[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    return;
  }

  uint64_t* bar_tma = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* bar_mma = bar_tma + 1;
  uint32_t* tmem_ptr = reinterpret_cast<uint32_t*>(smem + kOffTmemPtr);
  float* AF = reinterpret_cast<float*>(smem + kOffAF);
  float* TF = reinterpret_cast<float*>(smem + kOffTF);
  float* XS = reinterpret_cast<float*>(smem + kOffXS);
  float* gam = reinterpret_cast<float*>(smem + kOffGam);
  float* bet = reinterpret_cast<float*>(smem + kOffBeta);
  float* eg = reinterpret_cast<float*>(smem + kOffEG);

  if (warp == 0) {
    tmem_alloc(tmem_ptr, kTmCols);
    tmem_relinquish();
  }
  if (tid == 32) {
    mbar_init(bar_tma, 1);
    mbar_init(bar_mma, 1);
    fence_mbarrier_init();
    prefetch_tmap(&tm_q);
    prefetch_tmap(&tm_k);
    prefetch_tmap(&tm_v);
  }
  // Zero block Z of the stacked A operands.
  reinterpret_cast<uint4*>(smem + kOffTPZT + 16384)[tid] = make_uint4(0, 0, 0, 0);
  reinterpret_cast<uint4*>(smem + kOffTPZT + 16384)[tid + 256] = make_uint4(0, 0, 0, 0);

  // Initial state: thread (k = row, half) holds S^T[k][64*half + j] = S[64*half + j][k].
  float sreg[64];
#pragma unroll
  for (int j = 0; j < 64; ++j)
    sreg[j] = p.state ? p.state[sbase + static_cast<size_t>(64 * half + j) * kHeadDim + row] : 0.f;
  st_row_bf16(smem + kOffSB + half * 16384, row, sreg, 1.0f);
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_ptr;
  const uint32_t tm_lane = static_cast<uint32_t>(quad * 32) << 16;

  const uint32_t a_qkw = smem_u32(smem + kOffQKW);
  const uint32_t a_kb = smem_u32(smem + kOffKB);
  const uint32_t a_vb = smem_u32(smem + kOffVB);
  const uint32_t a_tpzt = smem_u32(smem + kOffTPZT);
  const uint32_t a_sb = smem_u32(smem + kOffSB);
  const uint32_t a_vn = smem_u32(smem + kOffVN);
  const uint32_t a_vnd = smem_u32(smem + kOffVND);

  const float A_neg = -expf(p.A_log[head]);
  const float dtb = p.dt_bias[head];

  uint32_t ph_tma = 0, ph_mma = 0;
  unsigned int fail = 0;
  const int nchunks = static_cast<int>((len + kChunk - 1) / kChunk);

  for (int ci = 0; ci < nchunks; ++ci) {
    const long long cstart = s0 + static_cast<long long>(ci) * kChunk;
    const int clen = static_cast<int>(min(static_cast<long long>(kChunk), s1 - cstart));

    // ---- 1. TMA: Q and K into the stacked operand, K and V tiles.
    if (tid == 0) {
      mbar_arrive_expect_tx(bar_tma, kTmaBytesPerChunk);
      const int t0 = static_cast<int>(cstart);
#pragma unroll
      for (int kb = 0; kb < 2; ++kb) {
        tma_load_3d(smem + kOffQKW + kb * 16384, &tm_q, bar_tma, kb * 64, hq, t0);
        tma_load_3d(smem + kOffQKW + kb * 16384 + 8192, &tm_k, bar_tma, kb * 64, hq, t0);
        tma_load_3d(smem + kOffKB + kb * 8192, &tm_k, bar_tma, kb * 64, hq, t0);
        tma_load_3d(smem + kOffVB + kb * 8192, &tm_v, bar_tma, kb * 64, head, t0);
      }
    }
    // ---- gates: log g, its inclusive prefix sum, beta (warp 1).
    if (warp == 1) {
      float lg[2], bt[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int pos = 2 * lane + e;
        if (pos < clen) {
          const size_t t = static_cast<size_t>(cstart + pos) * p.h_v + head;
          const float av = __bfloat162float(p.a[t]);
          const float bv = __bfloat162float(p.b[t]);
          lg[e] = A_neg * softplus20p(av + dtb);
          bt[e] = 1.0f / (1.0f + expf(-bv));
        } else {
          lg[e] = 0.f;
          bt[e] = 0.f;
        }
      }
      float x = lg[0] + lg[1];
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const float y = __shfl_up_sync(0xffffffffu, x, off);
        if (lane >= off) x += y;
      }
      const float excl = x - (lg[0] + lg[1]);
      const float g0 = excl + lg[0], g1 = g0 + lg[1];
      gam[2 * lane] = g0;
      gam[2 * lane + 1] = g1;
      eg[2 * lane] = expf(g0);
      eg[2 * lane + 1] = expf(g1);
      bet[2 * lane] = bt[0];
      bet[2 * lane + 1] = bt[1];
    }
    __syncthreads();
    {
      const bool ok = mbar_wait(bar_tma, ph_tma);
      if (__syncthreads_or(!ok)) { fail = kStatusTmaTimeout; break; }
      ph_tma ^= 1;
    }
    // Tail chunk: rows past the sequence end hold the next sequence's tokens
    // (or TMA zero fill); clear them so that 0 * (non-finite input) cannot reach S.
    if (clen < kChunk) {
      const int nrow = kChunk - clen;
      for (int e = tid; e < 8 * nrow * 8; e += kPrefillThreads) {
        const int reg = e / (nrow * 8);            // 8 row-blocks of 64 rows x 128 B
        const int r = clen + (e / 8) % nrow;
        const int cc = e & 7;
        const uint32_t base = (reg < 4) ? kOffQKW + (reg >> 1) * 16384 + (reg & 1) * 8192
                                        : (reg < 6 ? kOffKB : kOffVB) + (reg & 1) * 8192;
        *reinterpret_cast<uint4*>(smem + base + sw128_off(r, cc)) = make_uint4(0, 0, 0, 0);
      }
      fence_proxy_async_smem();
      __syncthreads();
    }

    // ---- 2. D_QK = [Q ; K] K^T.
    if (tid == 0) {
      tc_fence_after();
      const uint32_t idesc = idesc_bf16_f32(128, 64, 0, 0);
#pragma unroll
      for (int s = 0; s < 8; ++s) {
        const uint64_t ad = sdesc_sw128(a_qkw + (s >> 2) * 16384 + (s & 3) * 32, 16, 1024);
        const uint64_t bd = sdesc_sw128(a_kb + (s >> 2) * 8192 + (s & 3) * 32, 16, 1024);
        umma_bf16(tmem + kTmQK, ad, bd, idesc, s > 0 ? 1u : 0u);
      }
      umma_commit(bar_mma);
    }
    {
      const bool ok = mbar_wait(bar_mma, ph_mma);
      if (__syncthreads_or(!ok)) { fail = kStatusMmaTimeout; break; }
      ph_mma ^= 1;
    }
    tc_fence_after();

    // ---- 3. P (rows 0-63) to bf16, A (rows 64-127) to fp32.
    {
      float r[32];
      tmem_ld32(tmem + tm_lane + kTmQK + 32 * half, r);
      tmem_wait_ld();
      if (row < 64) {
        const int i = row;
        const float gi = gam[i];
#pragma unroll
        for (int jj = 0; jj < 32; ++jj) {
          const int j = 32 * half + jj;
          r[jj] = (j <= i && i < clen) ? r[jj] * expf(gi - gam[j]) : 0.f;
        }
        st_half_row_bf16(smem + kOffTPZT + 8192, i, 4 * half, r, 1.0f);
      } else {
        const int i = row - 64;
        const float gi = gam[i], nb = -bet[i];
#pragma unroll
        for (int jj = 0; jj < 32; ++jj) {
          const int j = 32 * half + jj;
          AF[i * kLdA + j] = (j < i && i < clen) ? nb * r[jj] * expf(gi - gam[j]) : 0.f;
        }
      }
    }
    tc_fence_before();
    __syncthreads();

    // ---- 4. T = (I - A)^{-1};  T' = T diag(beta e^gamma),  T_b = T diag(beta).
    solve_unit_lower(AF, TF, XS, tid);
    {
      const int i = tid >> 2, j0 = (tid & 3) * 16;
      float tp[16], tb[16];
#pragma unroll
      for (int jj = 0; jj < 16; ++jj) {
        const int j = j0 + jj;
        const float t = (j <= i) ? TF[i * kLdA + j] : 0.f;
        tb[jj] = t * bet[j];
        tp[jj] = tb[jj] * eg[j];
      }
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
        uint4 u, w;
        u.x = pack_bf16x2(tp[8 * h2 + 0], tp[8 * h2 + 1]);
        u.y = pack_bf16x2(tp[8 * h2 + 2], tp[8 * h2 + 3]);
        u.z = pack_bf16x2(tp[8 * h2 + 4], tp[8 * h2 + 5]);
        u.w = pack_bf16x2(tp[8 * h2 + 6], tp[8 * h2 + 7]);
        w.x = pack_bf16x2(tb[8 * h2 + 0], tb[8 * h2 + 1]);
        w.y = pack_bf16x2(tb[8 * h2 + 2], tb[8 * h2 + 3]);
        w.z = pack_bf16x2(tb[8 * h2 + 4], tb[8 * h2 + 5]);
        w.w = pack_bf16x2(tb[8 * h2 + 6], tb[8 * h2 + 7]);
        const uint32_t off = sw128_off(i, (tid & 3) * 2 + h2);
        *reinterpret_cast<uint4*>(smem + kOffTPZT + off) = u;           // T'
        *reinterpret_cast<uint4*>(smem + kOffTPZT + 24576 + off) = w;   // T_b
      }
    }
    fence_proxy_async_smem();
    __syncthreads();

    // ---- 5. D_W = [T' ; P] K,  D_UO = [Z ; T_b] V.
    if (tid == 0) {
      tc_fence_after();
      const uint32_t idesc = idesc_bf16_f32(128, 128, 0, 1);
#pragma unroll
      for (int s = 0; s < 4; ++s) {
        umma_bf16(tmem + kTmW, sdesc_sw128(a_tpzt + s * 32, 16, 1024),
                  sdesc_sw128(a_kb + s * 2048, 8192, 1024), idesc, s > 0 ? 1u : 0u);
      }
#pragma unroll
      for (int s = 0; s < 4; ++s) {
        umma_bf16(tmem + kTmUO, sdesc_sw128(a_tpzt + 16384 + s * 32, 16, 1024),
                  sdesc_sw128(a_vb + s * 2048, 8192, 1024), idesc, s > 0 ? 1u : 0u);
      }
      umma_commit(bar_mma);
    }
    {
      const bool ok = mbar_wait(bar_mma, ph_mma);
      if (__syncthreads_or(!ok)) { fail = kStatusMmaTimeout; break; }
      ph_mma ^= 1;
    }
    tc_fence_after();

    // ---- 6. -W into rows 64-127 of the stacked operand; Q <- e^gamma Q in rows 0-63.
    if (row < 64) {
      uint8_t* tile = smem + kOffQKW + half * 16384;
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        float r[32];
        tmem_ld32(tmem + tm_lane + kTmW + 64 * half + 32 * hh, r);
        tmem_wait_ld();
        st_half_row_bf16(tile, 64 + row, 4 * hh, r, -1.0f);
      }
    } else {
      const int c = row - 64;
      const float e = eg[c];
      uint8_t* tile = smem + kOffQKW + half * 16384;
#pragma unroll
      for (int cc = 0; cc < 8; ++cc) {
        uint4* ptr = reinterpret_cast<uint4*>(tile + sw128_off(c, cc));
        uint4 u = *ptr;
        uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
        for (int q2 = 0; q2 < 4; ++q2) {
          __nv_bfloat162 h2 = *reinterpret_cast<__nv_bfloat162*>(&w[q2]);
          float2 f = __bfloat1622float2(h2);
          w[q2] = pack_bf16x2(f.x * e, f.y * e);
        }
        *ptr = u;
      }
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();

    // ---- 7. D_UO += [e^g Q ; -W] S^T.
    if (tid == 0) {
      tc_fence_after();
      const uint32_t idesc = idesc_bf16_f32(128, 128, 0, 1);
#pragma unroll
      for (int s = 0; s < 8; ++s) {
        umma_bf16(tmem + kTmUO, sdesc_sw128(a_qkw + (s >> 2) * 16384 + (s & 3) * 32, 16, 1024),
                  sdesc_sw128(a_sb + s * 2048, 16384, 1024), idesc, 1u);
      }
      umma_commit(bar_mma);
    }
    {
      const bool ok = mbar_wait(bar_mma, ph_mma);
      if (__syncthreads_or(!ok)) { fail = kStatusMmaTimeout; break; }
      ph_mma ^= 1;
    }
    tc_fence_after();

    const float gam_last = gam[clen - 1];
    // ---- 8. v_new (rows 64-127) to bf16, plus its decayed copy.
    if (row >= 64) {
      const int c = row - 64;
      const float dec = (c < clen) ? expf(gam_last - gam[c]) : 0.f;
      const float keep = (c < clen) ? 1.f : 0.f;
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        float r[32];
        tmem_ld32(tmem + tm_lane + kTmUO + 64 * half + 32 * hh, r);
        tmem_wait_ld();
        st_half_row_bf16(smem + kOffVN + half * 8192, c, 4 * hh, r, keep);
        st_half_row_bf16(smem + kOffVND + half * 8192, c, 4 * hh, r, dec);
      }
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();

    // ---- 9. D_UO += [P ; Z] v_new;  D_S4 = K^T (v_new e^{gamma_last-gamma}).
    if (tid == 0) {
      tc_fence_after();
      const uint32_t idesc_o = idesc_bf16_f32(128, 128, 0, 1);
      const uint32_t idesc_s = idesc_bf16_f32(128, 128, 1, 1);
#pragma unroll
      for (int s = 0; s < 4; ++s) {
        umma_bf16(tmem + kTmUO, sdesc_sw128(a_tpzt + 8192 + s * 32, 16, 1024),
                  sdesc_sw128(a_vn + s * 2048, 8192, 1024), idesc_o, 1u);
      }
#pragma unroll
      for (int s = 0; s < 4; ++s) {
        umma_bf16(tmem + kTmS4, sdesc_sw128(a_kb + s * 2048, 8192, 1024),
                  sdesc_sw128(a_vnd + s * 2048, 8192, 1024), idesc_s, s > 0 ? 1u : 0u);
      }
      umma_commit(bar_mma);
    }
    {
      const bool ok = mbar_wait(bar_mma, ph_mma);
      if (__syncthreads_or(!ok)) { fail = kStatusMmaTimeout; break; }
      ph_mma ^= 1;
    }
    tc_fence_after();

    // ---- 10. Output rows (0-63) and the state update (all rows).
    if (row < 64) {
      __nv_bfloat16* orow = p.out + (static_cast<size_t>(cstart + row) * p.h_v + head) * kHeadDim +
                            64 * half;
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        float r[32];
        tmem_ld32(tmem + tm_lane + kTmUO + 64 * half + 32 * hh, r);
        tmem_wait_ld();
        if (row < clen) {
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) {
            uint4 u;
            u.x = pack_bf16x2(p.scale * r[8 * cc + 0], p.scale * r[8 * cc + 1]);
            u.y = pack_bf16x2(p.scale * r[8 * cc + 2], p.scale * r[8 * cc + 3]);
            u.z = pack_bf16x2(p.scale * r[8 * cc + 4], p.scale * r[8 * cc + 5]);
            u.w = pack_bf16x2(p.scale * r[8 * cc + 6], p.scale * r[8 * cc + 7]);
            *reinterpret_cast<uint4*>(orow + 32 * hh + 8 * cc) = u;
          }
        }
      }
    }
    {
      const float decay = expf(gam_last);
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        float r[32];
        tmem_ld32(tmem + tm_lane + kTmS4 + 64 * half + 32 * hh, r);
        tmem_wait_ld();
#pragma unroll
        for (int jj = 0; jj < 32; ++jj) sreg[32 * hh + jj] = fmaf(decay, sreg[32 * hh + jj], r[jj]);
      }
      st_row_bf16(smem + kOffSB + half * 16384, row, sreg, 1.0f);
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
  }

  if (fail) {
    // Give in-flight copies and UMMAs one more bounded wait before freeing TMEM.
    if (tid == 0) {
      atomicOr(p.status, fail);
      (void)mbar_wait(fail == kStatusTmaTimeout ? bar_tma : bar_mma,
                      fail == kStatusTmaTimeout ? ph_tma : ph_mma);
    }
    __syncthreads();
  } else {
#pragma unroll
    for (int j = 0; j < 64; ++j)
      p.new_state[sbase + static_cast<size_t>(64 * half + j) * kHeadDim + row] = sreg[j];
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, kTmCols);
}

}  // namespace gdn
