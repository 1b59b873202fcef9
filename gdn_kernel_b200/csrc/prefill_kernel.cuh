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
// The 64x64 triangular inverse: two 32x32 diagonal blocks by forward
// substitution on CUDA cores, one 32-level merge in 3xTF32 (fp32 accuracy).
//
// Pipelining: the next chunk's tiles are requested as soon as the buffer they
// land in has been consumed (V after the U product, Q and K after the S^T
// product, the K tile after the state-increment product), and the next chunk's
// gates are computed by a warp that is idle during the v_new epilogue.
//
// Every mbarrier wait is bounded; on a timeout the CTA records a status bit,
// stops at the end of the chunk, frees its TMEM and returns.
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
constexpr int kLdA = 68;                           // fp32 row pitch of A and T (16-byte rows)
constexpr uint32_t kOffAF = kOffVND + 16384;       // fp32 A [64][68]
constexpr uint32_t kOffTF = kOffAF + 64 * kLdA * 4;  // fp32 T [64][68]
constexpr uint32_t kOffXS = kOffTF + 64 * kLdA * 4;  // fp32 scratch of the solve, 32x40
constexpr uint32_t kGateFloats = 4 * 64;             // {gamma, beta, e^gamma, F}[64], F below
constexpr uint32_t kOffGate = kOffXS + 32 * 40 * 4;  // 2 gate buffers
constexpr uint32_t kOffBar = kOffGate + 2 * kGateFloats * 4;  // 5 mbarriers
constexpr uint32_t kOffTmemPtr = kOffBar + 48;
constexpr uint32_t kSmemUsed = kOffTmemPtr + 16;
constexpr uint32_t kPrefillSmem = kSmemUsed + 1024;  // slack to align the base

// TMEM column map (512 columns allocated, fp32 accumulators, lane = row).
constexpr uint32_t kTmQK = 0;
constexpr uint32_t kTmW = 64;
constexpr uint32_t kTmUO = 192;
constexpr uint32_t kTmS4 = 320;
constexpr uint32_t kTmCols = 512;

constexpr uint32_t kTileBytes = 8192;              // one 64 x 64 bf16 TMA box

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

// Store 32 fp32 values as chunks c0..c0+3 of a 128-byte bf16 row of a
// 128B-swizzled tile.
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

__device__ __forceinline__ void st_row_bf16(uint8_t* tile, uint32_t row, const float* x) {
  st_half_row_bf16(tile, row, 0, x, 1.0f);
  st_half_row_bf16(tile, row, 4, x + 32, 1.0f);
}

__device__ __forceinline__ void zero_half_row(uint8_t* tile, uint32_t row, uint32_t c0) {
#pragma unroll
  for (int cc = 0; cc < 4; ++cc)
    *reinterpret_cast<uint4*>(tile + sw128_off(row, c0 + cc)) = make_uint4(0, 0, 0, 0);
}

// Two 32-column TMEM loads in flight, then one wait.
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float (&r)[64]) {
  tmem_ld32(taddr, *reinterpret_cast<float(*)[32]>(r));
  tmem_ld32(taddr + 32, *reinterpret_cast<float(*)[32]>(r + 32));
  tmem_wait_ld();
}

// ---------------------------------------------------------------- triangular inverse
// 3xTF32 tensor-core products: x = x_hi + x_lo with both halves tf32, and
// a*b ~= a_hi*b_hi + a_hi*b_lo + a_lo*b_hi accumulated in fp32, which keeps the
// products at fp32-level accuracy.
__device__ __forceinline__ uint32_t to_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}

__device__ __forceinline__ void mma_tf32(float (&d)[4], const uint32_t (&a)[4],
                                         const uint32_t (&b)[2]) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// One 16x8 tile of D = L * R (L: 16 x 8*KSTEPS rows of pitch ldl; R: 8*KSTEPS x 8
// of pitch ldr), one warp, in single TF32 (10-bit mantissa operands, fp32
// accumulation).  Lane (g = lane/4, t = lane%4) receives
// D[g][2t], D[g][2t+1], D[g+8][2t], D[g+8][2t+1].
template <int KSTEPS>
__device__ __forceinline__ void mma_tile_tf32(float (&d)[4], const float* L, int ldl,
                                              const float* R, int ldr, int lane) {
  const int g = lane >> 2, t = lane & 3;
  float acc[KSTEPS][4];
#pragma unroll
  for (int ks = 0; ks < KSTEPS; ++ks) {
    const uint32_t a[4] = {to_tf32(L[g * ldl + 8 * ks + t]), to_tf32(L[(g + 8) * ldl + 8 * ks + t]),
                           to_tf32(L[g * ldl + 8 * ks + t + 4]),
                           to_tf32(L[(g + 8) * ldl + 8 * ks + t + 4])};
    const uint32_t b[2] = {to_tf32(R[(8 * ks + t) * ldr + g]), to_tf32(R[(8 * ks + t + 4) * ldr + g])};
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[ks][e] = 0.f;
    mma_tf32(acc[ks], a, b);
  }
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    float sum = 0.f;
#pragma unroll
    for (int ks = 0; ks < KSTEPS; ++ks) sum += acc[ks][e];
    d[e] = sum;
  }
}

// The same tile in 3xTF32 (operands split into a TF32 head and tail; fp32-level
// accuracy).
template <int KSTEPS>
__device__ __forceinline__ void mma_tile_3xtf32(float (&d)[4], const float* L, int ldl,
                                                const float* R, int ldr, int lane) {
  const int g = lane >> 2, t = lane & 3;
  // Every (k-step, split term) product gets its own accumulator, so the 3*KSTEPS
  // mma.sync issue back to back instead of forming one dependent chain.
  float acc[3 * KSTEPS][4];
#pragma unroll
  for (int ks = 0; ks < KSTEPS; ++ks) {
    const float av[4] = {L[g * ldl + 8 * ks + t], L[(g + 8) * ldl + 8 * ks + t],
                         L[g * ldl + 8 * ks + t + 4], L[(g + 8) * ldl + 8 * ks + t + 4]};
    const float bv[2] = {R[(8 * ks + t) * ldr + g], R[(8 * ks + t + 4) * ldr + g]};
    uint32_t ah[4], al[4], bh[2], bl[2];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      ah[e] = to_tf32(av[e]);
      al[e] = to_tf32(av[e] - __uint_as_float(ah[e]));
    }
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      bh[e] = to_tf32(bv[e]);
      bl[e] = to_tf32(bv[e] - __uint_as_float(bh[e]));
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[3 * ks][e] = acc[3 * ks + 1][e] = acc[3 * ks + 2][e] = 0.f;
    mma_tf32(acc[3 * ks], al, bh);
    mma_tf32(acc[3 * ks + 1], ah, bl);
    mma_tf32(acc[3 * ks + 2], ah, bh);
  }
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    float sum = 0.f;
#pragma unroll
    for (int q = 0; q < 3 * KSTEPS; ++q) sum += acc[q][e];
    d[e] = sum;
  }
}

// T'[i][j] = T[i][j] beta_j e^{gamma_j} and T_b[i][j] = T[i][j] beta_j, as bf16
// into the K-major swizzled tiles T' (TPZT + 0) and T_b (TPZT + 24 KiB).
__device__ __forceinline__ void st_tp_one(uint8_t* tpzt, int i, int j, float t, const float* bet,
                                          const float* eg) {
  const uint32_t off = sw128_off(i, j >> 3) + (j & 7) * 2;
  const float tb = t * bet[j];
  *reinterpret_cast<__nv_bfloat16*>(tpzt + 24576 + off) = __float2bfloat16(tb);
  *reinterpret_cast<__nv_bfloat16*>(tpzt + off) = __float2bfloat16(tb * eg[j]);
}

__device__ __forceinline__ void st_tp_pair(uint8_t* tpzt, int i, int j, float t0, float t1,
                                           const float* bet, const float* eg) {
  const uint32_t off = sw128_off(i, j >> 3) + (j & 7) * 2;   // j even: 4-byte aligned pair
  const float b0 = t0 * bet[j], b1 = t1 * bet[j + 1];
  *reinterpret_cast<uint32_t*>(tpzt + 24576 + off) = pack_bf16x2(b0, b1);
  *reinterpret_cast<uint32_t*>(tpzt + off) = pack_bf16x2(b0 * eg[j], b1 * eg[j + 1]);
}

// T = (I - A)^{-1} for the strictly lower 64x64 fp32 A (row pitch kLdA), by
// block doubling from 8x8 diagonal blocks:
//   1. the four 16x16 diagonal blocks T_bb = (I - A_bb)^{-1}: eight lanes of
//      warps 0 and 1 per 8x8 sub-block each solve one column by forward
//      substitution (8 dependent steps), then warps 0-3 form each block's
//      lower 8x8 part T_10 = T_11 (A_10 T_00) in fp32;
//   2. 16 -> 32: in each 32x32 diagonal block, T_10 = T_11 (A_10 T_00) as two
//      16x16 products (warps 0-3, one 16x8 tile each);
//   3. 32 -> 64: T_10 = T_11 (A_10 T_00) as two 32x32 products (all 8 warps).
// The block products run on the tensor cores in single TF32: T is only used
// through its bf16 copies (T', T_b), whose rounding (2^-9 relative) is coarser
// than TF32's (2^-11), and the fp32 T only feeds these products.
// Results go to T (fp32) and into the bf16 T' / T_b operand tiles.  The
// upper-right 32x32 blocks of the T' / T_b tiles are never written and must
// hold zeros; step 2 writes the zeros of the upper-right 16x16 blocks inside
// the diagonal 32x32 blocks (T' / T_b and the fp32 T that step 3 reads).
__device__ __forceinline__ void solve_unit_lower(const float* A, float* T, float* X, uint8_t* tpzt,
                                                 const float* bet, const float* eg, int tid) {
  const int warp = tid >> 5, lane = tid & 31;
  constexpr int kLdC = 40;    // pitch of the 32x32 scratch tile (conflict-free B fragments)
  if (warp < 2) {   // step 1a: 8x8 sub-block 4 warp + lane / 8, column lane % 8
    const int o = 8 * (4 * warp + (lane >> 3)), j = lane & 7;
    float x[8];
#pragma unroll
    for (int m = 0; m < 8; ++m) {
      // two partial sums keep the dependent chain short; the newest x enters last
      float acc[2] = {(m == j) ? 1.0f : 0.0f, 0.f};
      const float4* rp = reinterpret_cast<const float4*>(A + (o + m) * kLdA + o);
#pragma unroll
      for (int q = 0; q < (m + 3) / 4; ++q) {
        const float4 a4 = rp[q];
        const float av[4] = {a4.x, a4.y, a4.z, a4.w};
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if (4 * q + e < m) acc[e & 1] = fmaf(av[e], x[4 * q + e], acc[e & 1]);
      }
      x[m] = acc[0] + acc[1];
    }
#pragma unroll
    for (int m = 0; m < 8; ++m) {
      T[(o + m) * kLdA + o + j] = x[m];
      st_tp_one(tpzt, o + m, o + j, x[m], bet, eg);
    }
  } else if (warp < 4) {   // zeros of the upper-right 8x8 blocks inside the 16x16 diagonal blocks
    const int t = tid - 64;                                  // 64 threads
    const int blk = t >> 4, r = (t >> 1) & 7, part = t & 1;  // block, row, half row
    const int rr = 16 * blk + r, c0 = 16 * blk + 8 + 4 * part;
    *reinterpret_cast<float4*>(T + rr * kLdA + c0) = make_float4(0.f, 0.f, 0.f, 0.f);
    const uint32_t off = sw128_off(rr, (16 * blk + 8) / 8);
    *reinterpret_cast<uint2*>(tpzt + off + 8 * part) = make_uint2(0, 0);
    *reinterpret_cast<uint2*>(tpzt + 24576 + off + 8 * part) = make_uint2(0, 0);
  } else if (warp >= 4) {   // zeros of the upper-right 16x16 blocks inside the 32x32 diagonal blocks
    const int t = tid - 128;             // 128 threads
    const int blk = t >> 6, r = (t >> 2) & 15, part = t & 3;   // block, row, quarter row
    const int rr = 32 * blk + r, c0 = 32 * blk + 16 + 4 * part;
    *reinterpret_cast<float4*>(T + rr * kLdA + c0) = make_float4(0.f, 0.f, 0.f, 0.f);
    if (part < 2) {   // 16 bf16 = two 16-byte chunks per row and tile
      const uint32_t off = sw128_off(rr, (32 * blk + 16) / 8 + part);
      *reinterpret_cast<uint4*>(tpzt + off) = make_uint4(0, 0, 0, 0);
      *reinterpret_cast<uint4*>(tpzt + 24576 + off) = make_uint4(0, 0, 0, 0);
    }
  }
  if (warp < 4) {   // step 1b: 8 -> 16 in diagonal block b = warp: T_10 = T_11 (A_10 T_00), fp32
    named_sync(3, 128);   // warps 0-3: the 8x8 diagonal blocks and the zeros are written
    const int o = 16 * warp;
    const int r = lane >> 2, c = 2 * (lane & 3);             // rows r, columns c, c + 1
    float* Xb = X + warp * 64;                               // 8x8 scratch, pitch 8
    float y0 = 0.f, y1 = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float a = A[(o + 8 + r) * kLdA + o + k];
      y0 = fmaf(a, T[(o + k) * kLdA + o + c], y0);
      y1 = fmaf(a, T[(o + k) * kLdA + o + c + 1], y1);
    }
    Xb[r * 8 + c] = y0;
    Xb[r * 8 + c + 1] = y1;
    __syncwarp();
    float t0 = 0.f, t1 = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float tk = T[(o + 8 + r) * kLdA + o + 8 + k];
      t0 = fmaf(tk, Xb[k * 8 + c], t0);
      t1 = fmaf(tk, Xb[k * 8 + c + 1], t1);
    }
    T[(o + 8 + r) * kLdA + o + c] = t0;
    T[(o + 8 + r) * kLdA + o + c + 1] = t1;
    st_tp_pair(tpzt, o + 8 + r, o + c, t0, t1, bet, eg);
    // step 2a reads the 16x16 diagonal blocks warps 0-3 just completed; the
    // zeros of warps 4-7 are first read by step 3a, after the next CTA barrier
    named_sync(3, 128);
  }
  const int g = lane >> 2, t = lane & 3;
  if (warp < 4) {   // step 2a: X_B = A[32B+16.., 32B..] T[32B.., 32B..] (16x16, tile nt of block B)
    const int B = warp >> 1, nt = warp & 1, o = 32 * B;
    float d[4];
    mma_tile_tf32<2>(d, A + (o + 16) * kLdA + o, kLdA, T + o * kLdA + o + 8 * nt, kLdA, lane);
    float* Xp = X + 16 * B + 8 * nt;
    *reinterpret_cast<float2*>(Xp + g * kLdC + 2 * t) = make_float2(d[0], d[1]);
    *reinterpret_cast<float2*>(Xp + (g + 8) * kLdC + 2 * t) = make_float2(d[2], d[3]);
    // step 2b reads exactly the X_B tile this warp wrote
    __syncwarp();
  }
  if (warp < 4) {   // step 2b: T[32B+16.., 32B..] = T_11 X_B
    const int B = warp >> 1, nt = warp & 1, o = 32 * B;
    float d[4];
    mma_tile_tf32<2>(d, T + (o + 16) * kLdA + o + 16, kLdA, X + 16 * B + 8 * nt, kLdC, lane);
    const int row = o + 16 + g, col = o + 8 * nt + 2 * t;
    *reinterpret_cast<float2*>(T + row * kLdA + col) = make_float2(d[0], d[1]);
    *reinterpret_cast<float2*>(T + (row + 8) * kLdA + col) = make_float2(d[2], d[3]);
    st_tp_pair(tpzt, row, col, d[0], d[1], bet, eg);
    st_tp_pair(tpzt, row + 8, col, d[2], d[3], bet, eg);
  }
  __syncthreads();
  const int mt = warp >> 2, nt = warp & 3;
  {  // step 3a: X = A[32:64, 0:32] T[0:32, 0:32]
    float d[4];
    mma_tile_tf32<4>(d, A + (32 + 16 * mt) * kLdA, kLdA, T + 8 * nt, kLdA, lane);
    float* Xp = X + 16 * mt * kLdC + 8 * nt;
    *reinterpret_cast<float2*>(Xp + g * kLdC + 2 * t) = make_float2(d[0], d[1]);
    *reinterpret_cast<float2*>(Xp + (g + 8) * kLdC + 2 * t) = make_float2(d[2], d[3]);
  }
  // step 3b of column block nt reads the two 16-row halves warps nt and nt + 4 wrote
  named_sync(4 + nt, 64);
  {  // step 3b: T[32:64, 0:32] = T[32:64, 32:64] X  (only the bf16 tiles need it)
    float d[4];
    mma_tile_tf32<4>(d, T + (32 + 16 * mt) * kLdA + 32, kLdA, X + 8 * nt, kLdC, lane);
    const int row = 32 + 16 * mt + g, col = 8 * nt + 2 * t;
    st_tp_pair(tpzt, row, col, d[0], d[1], bet, eg);
    st_tp_pair(tpzt, row + 8, col, d[2], d[3], bet, eg);
  }
}

// Decay factors e^{gamma_i - gamma_j} of one row i over the 32 columns
// j = jb .. jb+31, zero where j > i or i >= clen.  gamma is non-increasing,
// so every factor is at most 1; each one is formed as a product of two
// factors that are also at most 1, through the end r = (j | 7) of j's
// 8-column sub-block when r <= i:
//   e^{gamma_i - gamma_j} = e^{gamma_i - gamma_r} * F[j],  F[j] = e^{gamma_r - gamma_j}
// (F per chunk from gate_finish).  Only the sub-block holding i itself needs
// direct exponentials.  Neither factor can overflow, and if one underflowed
// the exact product would too.  That is 11 exponentials per row in a
// diagonal 32x32 block and 4 in the block below it, instead of 32.
__device__ __forceinline__ void decay_row(int i, int jb, int clen, const float* gam,
                                          const float* fsub, float* f) {
  const float gi = gam[i];
  const int d = i - jb;   // >= 0 (the caller skips blocks above the diagonal)
  if (d >= 32) {          // the whole block lies below row i
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const float sb = __expf(gi - gam[jb + 8 * b + 7]);
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) f[8 * b + jj] = sb * fsub[jb + 8 * b + jj];
    }
  } else {                // diagonal block: i's own sub-block is sb, its offset in it dj
    const int sb = d >> 3, dj = d & 7;
    float e8[8];
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) e8[jj] = __expf(gi - gam[jb + 8 * sb + jj]);
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const float s_b = b < 3 ? __expf(gi - gam[jb + 8 * b + 7]) : 0.f;   // used when b < sb
#pragma unroll
      for (int jj = 0; jj < 8; ++jj)
        f[8 * b + jj] = b < sb ? s_b * fsub[jb + 8 * b + jj] : (b == sb && jj <= dj ? e8[jj] : 0.f);
    }
  }
  if (i >= clen) {
#pragma unroll
    for (int jj = 0; jj < 32; ++jj) f[jj] = 0.f;
  }
}

// P (rows 0-63 of D_QK) to the bf16 P tile and A (rows 64-127) to fp32, for
// the TMEM lane `row` of this thread and the 32 columns of its `half`:
//   P_ij = (QK^T)_ij e^{gamma_i - gamma_j}          (j <= i < clen, else 0)
//   A_ij = -beta_i (KK^T)_ij e^{gamma_i - gamma_j}  (j < i < clen, else 0)
// A 32-column tile that lies wholly above the diagonal skips the exponentials.
__device__ __forceinline__ void pa_epilogue(uint32_t tm_qk, int row, int half, int quad, int clen,
                                            const float* gam, const float* bet, const float* fsub,
                                            uint8_t* ptile, float* AF) {
  const int i = row & 63;
  const bool upper = half == 1 && (quad & 1) == 0;   // rows 0-31 x cols 32-63
  if (upper) {
    if (row < 64) zero_half_row(ptile, i, 4);
    return;
  }
  float r[32], f[32];
  tmem_ld32(tm_qk + 32 * half, r);
  decay_row(i, 32 * half, clen, gam, fsub, f);   // overlaps the TMEM load
  tmem_wait_ld();
  if (row < 64) {
#pragma unroll
    for (int jj = 0; jj < 32; ++jj) r[jj] *= f[jj];
    st_half_row_bf16(ptile, i, 4 * half, r, 1.0f);
  } else {
    const float nb = -bet[i];
    float* arow = AF + i * kLdA + 32 * half;
#pragma unroll
    for (int jj = 0; jj < 32; jj += 4) {
      float4 o;
      const int j = 32 * half + jj;
      o.x = j + 0 < i ? nb * r[jj + 0] * f[jj + 0] : 0.f;
      o.y = j + 1 < i ? nb * r[jj + 1] * f[jj + 1] : 0.f;
      o.z = j + 2 < i ? nb * r[jj + 2] * f[jj + 2] : 0.f;
      o.w = j + 3 < i ? nb * r[jj + 3] * f[jj + 3] : 0.f;
      *reinterpret_cast<float4*>(arow + jj) = o;
    }
  }
}

// Q <- e^gamma Q in place on one 128-byte row of one K-column of a stacked
// K-major tile.
__device__ __forceinline__ void scale_q_row(uint8_t* tile, int c, float e) {
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

// Q'[c] = e Q[c] - pw in place on the 64 columns of one 128-byte row of a
// K-major swizzled tile (pw: fp32, the same 64 columns).
__device__ __forceinline__ void qprime_row(uint8_t* tile, int c, float e, const float* pw) {
#pragma unroll
  for (int cc = 0; cc < 8; ++cc) {
    uint4* ptr = reinterpret_cast<uint4*>(tile + sw128_off(c, cc));
    uint4 u = *ptr;
    uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
    for (int q2 = 0; q2 < 4; ++q2) {
      const float2 f = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&w[q2]));
      w[q2] = pack_bf16x2(fmaf(e, f.x, -pw[8 * cc + 2 * q2]), fmaf(e, f.y, -pw[8 * cc + 2 * q2 + 1]));
    }
    *ptr = u;
  }
}

// Gates of one chunk (one warp, two positions per lane).  gate_inputs loads
// a and b (issued early, so their latency hides behind other work);
// gate_finish forms log g, its inclusive prefix sum gamma, e^gamma, beta and
// F[j] = e^{gamma_{j|7} - gamma_j} (the decay from j to the end of its
// 8-position sub-block, used by decay_row).
// Positions past the sequence end get log g = 0 and beta = 0.
// The inputs stay bf16 until gate_finish: a conversion here would make the
// warp wait for the loads where they are issued.
struct GateIn {
  __nv_bfloat16 a[2], b[2];
  bool valid[2];
};

__device__ __forceinline__ GateIn gate_inputs(const PrefillParams& p, long long cstart, int clen,
                                              int head, int lane) {
  GateIn g;
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const int pos = 2 * lane + e;
    g.valid[e] = pos < clen;
    if (g.valid[e]) {
      const size_t t = static_cast<size_t>(cstart + pos) * p.h_v + head;
      g.a[e] = p.a[t];
      g.b[e] = p.b[t];
    } else {
      g.a[e] = g.b[e] = __float2bfloat16(0.f);
    }
  }
  return g;
}

__device__ __forceinline__ void gate_finish(const GateIn& g, float A_neg, float dtb, int lane,
                                            float* gam, float* bet, float* eg, float* fsub) {
  float lg[2], bt[2];
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    lg[e] = g.valid[e] ? A_neg * softplus20p(__bfloat162float(g.a[e]) + dtb) : 0.f;
    bt[e] = g.valid[e] ? 1.0f / (1.0f + expf(-__bfloat162float(g.b[e]))) : 0.f;
  }
  float x = lg[0] + lg[1];
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const float y = __shfl_up_sync(0xffffffffu, x, off);
    if (lane >= off) x += y;
  }
  const float g0 = (x - (lg[0] + lg[1])) + lg[0], g1 = g0 + lg[1];
  gam[2 * lane] = g0;
  gam[2 * lane + 1] = g1;
  eg[2 * lane] = expf(g0);
  eg[2 * lane + 1] = expf(g1);
  // position 2 lane | 7 ends this lane's sub-block; lane (lane | 3) holds it as g1
  const float gend = __shfl_sync(0xffffffffu, g1, lane | 3);
  fsub[2 * lane] = expf(gend - g0);
  fsub[2 * lane + 1] = expf(gend - g1);
  bet[2 * lane] = bt[0];
  bet[2 * lane + 1] = bt[1];
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
  if (s0 < 0 || s1 < s0 || s1 > p.total_tokens) {
    if (tid == 0) atomicOr(p.status, kStatusBadSeqlens);   // treated as an empty sequence
    s0 = s1 = 0;
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

  uint64_t* bar_q = reinterpret_cast<uint64_t*>(smem + kOffBar);   // Q + K copy -> QKW
  uint64_t* bar_k = bar_q + 1;                                      // K -> KB
  uint64_t* bar_v = bar_q + 2;                                      // V -> VB
  uint64_t* bar_mma = bar_q + 3;                                    // UMMA groups
  uint64_t* bar_mma2 = bar_q + 4;                                   // second UMMA group of a step
  uint32_t* tmem_ptr = reinterpret_cast<uint32_t*>(smem + kOffTmemPtr);
  float* AF = reinterpret_cast<float*>(smem + kOffAF);
  float* TF = reinterpret_cast<float*>(smem + kOffTF);
  float* XS = reinterpret_cast<float*>(smem + kOffXS);
  float* gate_base = reinterpret_cast<float*>(smem + kOffGate);

  const float A_neg = -expf(p.A_log[head]);
  const float dtb = p.dt_bias[head];
  const int nchunks = static_cast<int>((len + kChunk - 1) / kChunk);

  auto load_q = [&](long long cstart) {
    mbar_arrive_expect_tx(bar_q, 4 * kTileBytes);
    const int t0 = static_cast<int>(cstart);
#pragma unroll
    for (int kb = 0; kb < 2; ++kb) {
      tma_load_3d(smem + kOffQKW + kb * 16384, &tm_q, bar_q, kb * 64, hq, t0);
      tma_load_3d(smem + kOffQKW + kb * 16384 + 8192, &tm_k, bar_q, kb * 64, hq, t0);
    }
  };
  auto load_k = [&](long long cstart) {
    mbar_arrive_expect_tx(bar_k, 2 * kTileBytes);
#pragma unroll
    for (int kb = 0; kb < 2; ++kb)
      tma_load_3d(smem + kOffKB + kb * 8192, &tm_k, bar_k, kb * 64, hq, static_cast<int>(cstart));
  };
  auto load_v = [&](long long cstart) {
    mbar_arrive_expect_tx(bar_v, 2 * kTileBytes);
#pragma unroll
    for (int kb = 0; kb < 2; ++kb)
      tma_load_3d(smem + kOffVB + kb * 8192, &tm_v, bar_v, kb * 64, head, static_cast<int>(cstart));
  };

  if (warp == 0) {
    tmem_alloc(tmem_ptr, kTmCols);
    tmem_relinquish();
  }
  if (tid == 32) {
    for (int i = 0; i < 5; ++i) mbar_init(bar_q + i, 1);
    fence_mbarrier_init();
    prefetch_tmap(&tm_q);
    prefetch_tmap(&tm_k);
    prefetch_tmap(&tm_v);
  }
  // Zero the whole T' | P | Z | T_b region: Z stays zero, and the upper-right
  // blocks of T' and T_b are never written by the solve.
  for (int i = tid; i < 32768 / 16; i += kPrefillThreads)
    reinterpret_cast<uint4*>(smem + kOffTPZT)[i] = make_uint4(0, 0, 0, 0);
  __syncthreads();
  if (tid == 0) {   // chunk 0 tiles
    load_q(s0);
    load_k(s0);
    load_v(s0);
  }
  if (warp == 1) {
    const GateIn g0 = gate_inputs(p, s0, static_cast<int>(min(static_cast<long long>(kChunk), len)),
                                  head, lane);
    gate_finish(g0, A_neg, dtb, lane, gate_base, gate_base + 64, gate_base + 128, gate_base + 192);
  }

  // Initial state: thread (k = row, half) holds S^T[k][64*half + j] = S[64*half + j][k].
  float sreg[64];
#pragma unroll
  for (int j = 0; j < 64; ++j)
    sreg[j] = p.state ? p.state[sbase + static_cast<size_t>(64 * half + j) * kHeadDim + row] : 0.f;
  st_row_bf16(smem + kOffSB + half * 16384, row, sreg);
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

  uint32_t ph = 0;            // phase of the per-chunk barriers (each completes once per chunk)
  uint32_t ph_mma = 0, ph_mma2 = 0;
  GateIn next_gates;          // warp 1: the next chunk's a, b, loaded one chunk ahead
  bool failed = false;        // this thread saw a wait run out
  unsigned int fail_code = 0;
  uint64_t* fail_bar = nullptr;
  uint32_t fail_parity = 0;
  auto wait = [&](uint64_t* bar, uint32_t parity, unsigned int code) {
    if (!mbar_wait(bar, parity)) {
      if (!failed) {
        fail_bar = bar;
        fail_parity = parity;
      }
      failed = true;
      fail_code |= code;
    }
  };
  auto mma_done = [&]() {
    wait(bar_mma, ph_mma, kStatusMmaTimeout);
    ph_mma ^= 1;
    tc_fence_after();
  };
  auto mma2_done = [&]() {
    wait(bar_mma2, ph_mma2, kStatusMmaTimeout);
    ph_mma2 ^= 1;
    tc_fence_after();
  };

  for (int ci = 0; ci < nchunks; ++ci) {
    const long long cstart = s0 + static_cast<long long>(ci) * kChunk;
    const int clen = static_cast<int>(min(static_cast<long long>(kChunk), s1 - cstart));
    const bool has_next = ci + 1 < nchunks;
    const long long nstart = cstart + kChunk;
    const float* gam = gate_base + (ci & 1) * kGateFloats;
    const float* bet = gam + 64;
    const float* eg = gam + 128;

    // ---- 1. wait for this chunk's Q/K tiles (requested during the previous chunk).
    if (warp == 1 && has_next)
      next_gates = gate_inputs(p, nstart,
                               static_cast<int>(min(static_cast<long long>(kChunk), s1 - nstart)),
                               head, lane);
    wait(bar_q, ph, kStatusTmaTimeout);
    wait(bar_k, ph, kStatusTmaTimeout);
    if (clen < kChunk) {
      // Tail chunk: rows past the sequence end hold the next sequence's tokens
      // (or TMA zero fill); clear them so that 0 * (non-finite input) cannot reach S.
      wait(bar_v, ph, kStatusTmaTimeout);
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
    mma_done();

    // ---- 3. P (rows 0-63) to bf16, A (rows 64-127) to fp32.
    pa_epilogue(tmem + tm_lane + kTmQK, row, half, quad, clen, gam, bet, gam + 192,
                smem + kOffTPZT + 8192, AF);
    tc_fence_before();
    __syncthreads();

    // ---- 4. T = (I - A)^{-1};  T' = T diag(beta e^gamma),  T_b = T diag(beta).
    solve_unit_lower(AF, TF, XS, smem + kOffTPZT, bet, eg, tid);
    fence_proxy_async_smem();
    __syncthreads();

    // ---- 5. D_W = [T' ; P] K,  D_UO = [Z ; T_b] V.
    if (tid == 0) {
      if (clen == kChunk) wait(bar_v, ph, kStatusTmaTimeout);
      tc_fence_after();
      const uint32_t idesc = idesc_bf16_f32(128, 128, 0, 1);
#pragma unroll
      for (int s = 0; s < 4; ++s) {
        umma_bf16(tmem + kTmW, sdesc_sw128(a_tpzt + s * 32, 16, 1024),
                  sdesc_sw128(a_kb + s * 2048, 8192, 1024), idesc, s > 0 ? 1u : 0u);
      }
      umma_commit(bar_mma);    // W first: its epilogue starts while U is computed
#pragma unroll
      for (int s = 0; s < 4; ++s) {
        umma_bf16(tmem + kTmUO, sdesc_sw128(a_tpzt + 16384 + s * 32, 16, 1024),
                  sdesc_sw128(a_vb + s * 2048, 8192, 1024), idesc, s > 0 ? 1u : 0u);
      }
      umma_commit(bar_mma2);
    }

    // ---- 6. -W into rows 64-127 of the stacked operand; Q <- e^gamma Q in rows 0-63.
    if (row < 64) {
      mma_done();
      float r[64];
      tmem_ld64(tmem + tm_lane + kTmW + 64 * half, r);
      uint8_t* tile = smem + kOffQKW + half * 16384;
      st_half_row_bf16(tile, 64 + row, 0, r, -1.0f);
      st_half_row_bf16(tile, 64 + row, 4, r + 32, -1.0f);
    } else {
      const int c = row - 64;
      scale_q_row(smem + kOffQKW + half * 16384, c, eg[c]);
      ph_mma ^= 1;   // this thread does not read D_W
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();

    // ---- 7. D_UO += [e^g Q ; -W] S^T.
    if (tid == 0) {
      mma2_done();                                // U is in D_UO
      if (has_next) load_v(nstart);               // VB is free once the U product completed
      const uint32_t idesc = idesc_bf16_f32(128, 128, 0, 1);
#pragma unroll
      for (int s = 0; s < 8; ++s) {
        umma_bf16(tmem + kTmUO, sdesc_sw128(a_qkw + (s >> 2) * 16384 + (s & 3) * 32, 16, 1024),
                  sdesc_sw128(a_sb + s * 2048, 16384, 1024), idesc, 1u);
      }
      umma_commit(bar_mma);
    }
    if (tid != 0) ph_mma2 ^= 1;   // the U group was consumed by thread 0 alone
    mma_done();
    if (tid == 0 && has_next) load_q(nstart);   // QKW is free once the S^T product completed

    const float gam_last = gam[clen - 1];
    // ---- 8. v_new (rows 64-127) to bf16 plus its decayed copy; meanwhile warp 1
    // computes the next chunk's gates into the other gate buffer.
    if (row >= 64) {
      const int c = row - 64;
      const float dec = (c < clen) ? __expf(gam_last - gam[c]) : 0.f;
      const float keep = (c < clen) ? 1.f : 0.f;
      float r[64];
      tmem_ld64(tmem + tm_lane + kTmUO + 64 * half, r);
      st_half_row_bf16(smem + kOffVN + half * 8192, c, 0, r, keep);
      st_half_row_bf16(smem + kOffVN + half * 8192, c, 4, r + 32, keep);
      st_half_row_bf16(smem + kOffVND + half * 8192, c, 0, r, dec);
      st_half_row_bf16(smem + kOffVND + half * 8192, c, 4, r + 32, dec);
    } else if (warp == 1 && has_next) {
      float* ng = gate_base + ((ci + 1) & 1) * kGateFloats;
      gate_finish(next_gates, A_neg, dtb, lane, ng, ng + 64, ng + 128, ng + 192);
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
        umma_bf16(tmem + kTmS4, sdesc_sw128(a_kb + s * 2048, 8192, 1024),
                  sdesc_sw128(a_vnd + s * 2048, 8192, 1024), idesc_s, s > 0 ? 1u : 0u);
      }
      umma_commit(bar_mma);    // the state increment first: it is on the chunk chain
#pragma unroll
      for (int s = 0; s < 4; ++s) {
        umma_bf16(tmem + kTmUO, sdesc_sw128(a_tpzt + 8192 + s * 32, 16, 1024),
                  sdesc_sw128(a_vn + s * 2048, 8192, 1024), idesc_o, 1u);
      }
      umma_commit(bar_mma2);
    }
    mma_done();
    if (tid == 0 && has_next) load_k(nstart);   // KB is free once the state product completed

    // ---- 10. State update (all rows) and output rows (0-63).
    {
      const float decay = __expf(gam_last);
      float r[64];
      tmem_ld64(tmem + tm_lane + kTmS4 + 64 * half, r);
#pragma unroll
      for (int jj = 0; jj < 64; ++jj) sreg[jj] = fmaf(decay, sreg[jj], r[jj]);
      st_row_bf16(smem + kOffSB + half * 16384, row, sreg);
    }
    if (row < 64) {
      mma2_done();
      float r[64];
      tmem_ld64(tmem + tm_lane + kTmUO + 64 * half, r);
      if (row < clen) {
        __nv_bfloat16* orow = p.out + (static_cast<size_t>(cstart + row) * p.h_v + head) *
                                          kHeadDim + 64 * half;
#pragma unroll
        for (int cc = 0; cc < 8; ++cc) {
          uint4 u;
          u.x = pack_bf16x2(p.scale * r[8 * cc + 0], p.scale * r[8 * cc + 1]);
          u.y = pack_bf16x2(p.scale * r[8 * cc + 2], p.scale * r[8 * cc + 3]);
          u.z = pack_bf16x2(p.scale * r[8 * cc + 4], p.scale * r[8 * cc + 5]);
          u.w = pack_bf16x2(p.scale * r[8 * cc + 6], p.scale * r[8 * cc + 7]);
          *reinterpret_cast<uint4*>(orow + 8 * cc) = u;
        }
      }
    } else {
      ph_mma2 ^= 1;   // these rows hold no output
    }
    fence_proxy_async_smem();
    tc_fence_before();
    ph ^= 1;
    if (__syncthreads_or(failed)) break;
  }

  const bool any_fail = __syncthreads_or(failed);
  if (any_fail) {
    if (failed) {
      atomicOr(p.status, fail_code);
      // one more bounded wait for the copy or UMMA that did not arrive
      if (lane == 0) (void)mbar_wait(fail_bar, fail_parity);
    }
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
