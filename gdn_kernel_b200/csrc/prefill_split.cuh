// Two-stage chunked prefill: the S-independent work of every (chunk, v-head)
// runs fully parallel in one kernel, and the sequential state recurrence runs
// in a second kernel that only does the S-dependent products.
//
//   gdn_chunk_table_kernel   cu_seqlens -> per-sequence chunk offsets and a flat
//                            table of (sequence, chunk start, chunk length).
//   gdn_prefill_prep_kernel  one CTA per (chunk, v-head), two CTAs per SM:
//                            gates, D_QK = [Q;K]K^T, P and A, the triangular
//                            inverse, D_W = [T';P]K, then -W and e^gamma Q.  It
//                            stores the bf16 operand tiles exactly as they sit
//                            in shared memory (128B-swizzled "tile images"):
//                            [e^g Q ; -W] (32 KiB), P (8 KiB), T_b (8 KiB), gamma.
//   gdn_prefill_chain_kernel one CTA per (sequence, v-head, 64-column V slice):
//                            per chunk, bulk-copies the tile images back into
//                            shared memory (double-buffered, two chunks ahead),
//                            and runs
//                              D_UO  = [Z ; T_b] V_s + [e^g Q ; -W] S_s^T
//                              v_new = rows 64-127 of D_UO
//                              D_S4  = K^T (v_new e^{gamma_last-gamma})
//                              D_UO += [P ; Z] v_new      (rows 0-63: output)
//                              S_s^T = e^{gamma_last} S_s^T + D_S4
//                            The output rows of a chunk are written while the
//                            tensor core already runs the next chunk.
//
// The arithmetic per element is that of the single-kernel path (same operand
// tiles, same accumulation), so both paths agree with the oracle to the same
// tolerance.  The workspace holds the tables and one 49 KiB record per
// (chunk, v-head); it is caller-provided (gdn_b200_prefill_workspace_size),
// 256-byte aligned (records sit at 1 KiB multiples from its start).
#pragma once

#include "prefill_kernel.cuh"

namespace gdn {

struct ChunkInfo {
  int seq;
  int clen;           // 0 marks a table slot past the last chunk
  long long cstart;
};

// Record of one (chunk, v-head) in the workspace.
constexpr uint32_t kRecOffQW = 0;          // [e^g Q ; -W] tile image, 32 KiB
constexpr uint32_t kRecOffP = 32768;       // P tile image, 8 KiB
constexpr uint32_t kRecOffTb = 40960;      // T_b tile image, 8 KiB
constexpr uint32_t kRecOffGam = 49152;     // gamma[64], 256 B
constexpr uint32_t kRecBytes = 50176;      // 49 KiB (keeps records 1 KiB aligned)

struct SplitLayout {
  size_t off_header, off_seq, off_table, off_rec, total;
  long long max_chunks;
};

__host__ __device__ inline SplitLayout split_layout(long long num_seqs, long long total_tokens,
                                                    int h_v) {
  SplitLayout L;
  L.max_chunks = (total_tokens + kChunk - 1) / kChunk + num_seqs;
  auto up = [](size_t x, size_t a) { return (x + a - 1) / a * a; };
  L.off_header = 0;
  L.off_seq = 256;
  L.off_table = up(L.off_seq + static_cast<size_t>(num_seqs + 1) * 4, 1024);
  L.off_rec = up(L.off_table + static_cast<size_t>(L.max_chunks) * sizeof(ChunkInfo), 1024);
  L.total = L.off_rec + static_cast<size_t>(L.max_chunks) * h_v * kRecBytes;
  return L;
}

struct SplitParams {
  PrefillParams base;
  int* header;            // [0] = total chunks
  int* seq_off;           // [N + 1] first chunk of each sequence
  ChunkInfo* table;       // [max_chunks]
  uint8_t* records;       // [max_chunks][H_v] x kRecBytes
  int num_seqs;
  int max_chunks;
};

// ---------------------------------------------------------------- chunk table
constexpr int kTableThreads = 1024;

__global__ void __launch_bounds__(kTableThreads) gdn_chunk_table_kernel(SplitParams sp) {
  __shared__ int warp_sums[32];
  __shared__ int carry_s;
  const PrefillParams& p = sp.base;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) carry_s = 0;
  __syncthreads();
  for (int base = 0; base < sp.num_seqs; base += kTableThreads) {
    const int i = base + tid;
    int n = 0;
    long long s0 = 0, s1 = 0;
    if (i < sp.num_seqs) {
      s0 = load_cu(p, i);
      s1 = load_cu(p, i + 1);
      if (s0 < 0 || s1 > p.total_tokens || s0 > p.total_tokens) {
        atomicOr(p.status, kStatusBadSeqlens);   // treated as an empty sequence
        s1 = s0;
      }
      n = s1 > s0 ? static_cast<int>((s1 - s0 + kChunk - 1) / kChunk) : 0;
    }
    int x = n;   // inclusive warp scan
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, off);
      if (lane >= off) x += y;
    }
    if (lane == 31) warp_sums[warp] = x;
    __syncthreads();
    if (warp == 0) {
      int w = warp_sums[lane];
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, w, off);
        if (lane >= off) w += y;
      }
      warp_sums[lane] = w;   // inclusive over warps
    }
    __syncthreads();
    const int excl = carry_s + (warp > 0 ? warp_sums[warp - 1] : 0) + x - n;
    if (i < sp.num_seqs) {
      sp.seq_off[i] = excl;
      for (int k = 0; k < n; ++k) {
        ChunkInfo c;
        c.seq = i;
        c.cstart = s0 + static_cast<long long>(k) * kChunk;
        c.clen = static_cast<int>(min(static_cast<long long>(kChunk), s1 - c.cstart));
        sp.table[excl + k] = c;
      }
    }
    __syncthreads();
    if (tid == kTableThreads - 1) carry_s = excl + n;
    __syncthreads();
  }
  if (tid == 0) {
    sp.seq_off[sp.num_seqs] = carry_s;
    sp.header[0] = carry_s;
  }
  // Table slots past the last chunk get clen = 0: the prep kernel's CTAs for
  // them read one entry and exit.
  for (int i = carry_s + tid; i < sp.max_chunks; i += kTableThreads) {
    ChunkInfo c;
    c.seq = -1;
    c.clen = 0;
    c.cstart = 0;
    sp.table[i] = c;
  }
}

// ---------------------------------------------------------------- bulk copies
// 1-D bulk copies (no tensor map; 16-byte aligned addresses and sizes).
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void bulk_store(void* gdst, const void* smem_src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gdst),
               "r"(smem_u32(smem_src)), "r"(bytes)
               : "memory");
}

// Commit this thread's bulk stores and wait until their shared-memory sources
// have been read (the global writes complete before the kernel does).
__device__ __forceinline__ void bulk_commit_and_wait_read() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}

// ---------------------------------------------------------------- prep kernel
constexpr uint32_t kP1OffQKW = 0;                      // 32 KiB [Q;K] then [e^g Q; -W]
constexpr uint32_t kP1OffTPZT = 32768;                 // 32 KiB T' | P | (unused) | T_b
constexpr uint32_t kP1OffAF = 65536;
constexpr uint32_t kP1OffTF = kP1OffAF + 64 * kLdA * 4;
constexpr uint32_t kP1OffXS = kP1OffTF + 64 * kLdA * 4;
constexpr uint32_t kP1OffGate = kP1OffXS + 32 * 40 * 4;   // gamma, beta, e^gamma [64]
constexpr uint32_t kP1OffBar = kP1OffGate + 768;
constexpr uint32_t kP1OffTmemPtr = kP1OffBar + 16;
constexpr uint32_t kP1Smem = kP1OffTmemPtr + 16 + 1024;
constexpr uint32_t kP1TmQK = 0;       // 64 columns
constexpr uint32_t kP1TmW = 64;       // 128 columns
constexpr uint32_t kP1TmCols = 256;

__global__ void __launch_bounds__(kPrefillThreads, 2)
    gdn_prefill_prep_kernel(const __grid_constant__ CUtensorMap tm_q,
                            const __grid_constant__ CUtensorMap tm_k, const SplitParams sp) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const PrefillParams& p = sp.base;
  const int gc = blockIdx.x, head = blockIdx.y;
  const ChunkInfo info = sp.table[gc];
  if (info.clen <= 0) return;   // slot past the last chunk
  const int clen = info.clen;
  const long long cstart = info.cstart;
  const int hq = head / (p.h_v / p.h_qk);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quad = warp & 3, half = warp >> 2, row = quad * 32 + lane;

  uint64_t* bar_tma = reinterpret_cast<uint64_t*>(smem + kP1OffBar);
  uint64_t* bar_mma = bar_tma + 1;
  uint32_t* tmem_ptr = reinterpret_cast<uint32_t*>(smem + kP1OffTmemPtr);
  float* AF = reinterpret_cast<float*>(smem + kP1OffAF);
  float* TF = reinterpret_cast<float*>(smem + kP1OffTF);
  float* XS = reinterpret_cast<float*>(smem + kP1OffXS);
  float* gam = reinterpret_cast<float*>(smem + kP1OffGate);
  float* bet = gam + 64;
  float* eg = gam + 128;
  uint8_t* tpzt = smem + kP1OffTPZT;

  if (warp == 0) {
    tmem_alloc(tmem_ptr, kP1TmCols);
    tmem_relinquish();
  }
  if (tid == 32) {
    mbar_init(bar_tma, 1);
    mbar_init(bar_mma, 1);
    fence_mbarrier_init();
    prefetch_tmap(&tm_q);
    prefetch_tmap(&tm_k);
  }
  // The solve never writes the upper-right 32x32 blocks of the T' and T_b
  // tiles (rows 0-31, 16-byte chunks 4-7): they hold zeros.
  {
    const int r = tid >> 3, c = 4 + ((tid >> 1) & 3), t = tid & 1;
    *reinterpret_cast<uint4*>(tpzt + 24576 * t + sw128_off(r, c)) = make_uint4(0, 0, 0, 0);
  }
  __syncthreads();
  if (tid == 0) {
    mbar_arrive_expect_tx(bar_tma, 4 * kTileBytes);
    const int t0 = static_cast<int>(cstart);
#pragma unroll
    for (int kb = 0; kb < 2; ++kb) {
      tma_load_3d(smem + kP1OffQKW + kb * 16384, &tm_q, bar_tma, kb * 64, hq, t0);
      tma_load_3d(smem + kP1OffQKW + kb * 16384 + 8192, &tm_k, bar_tma, kb * 64, hq, t0);
    }
  }
  if (warp == 1) {
    const GateIn g = gate_inputs(p, cstart, clen, head, lane);
    gate_finish(g, -expf(p.A_log[head]), p.dt_bias[head], lane, gam, bet, eg);
  }
  const bool ok = mbar_wait(bar_tma, 0);
  unsigned int code = ok ? 0u : kStatusTmaTimeout;
  if (clen < kChunk) {   // rows past the sequence end: zero Q and K rows
    const int nrow = kChunk - clen;
    for (int e = tid; e < 4 * nrow * 8; e += kPrefillThreads) {
      const int reg = e / (nrow * 8);
      const int r = clen + (e / 8) % nrow;
      const uint32_t base = kP1OffQKW + (reg >> 1) * 16384 + (reg & 1) * 8192;
      *reinterpret_cast<uint4*>(smem + base + sw128_off(r, e & 7)) = make_uint4(0, 0, 0, 0);
    }
  }
  fence_proxy_async_smem();
  tc_fence_before();
  const bool fail0 = __syncthreads_or(!ok);
  tc_fence_after();
  const uint32_t tmem = *tmem_ptr;
  const uint32_t tm_lane = static_cast<uint32_t>(quad * 32) << 16;
  const uint32_t a_qkw = smem_u32(smem + kP1OffQKW);
  const uint32_t a_tpzt = smem_u32(tpzt);

  if (!fail0) {
    // D_QK = [Q ; K] K^T, with K (rows 64-127 of the stacked tile) as the B operand.
    if (tid == 0) {
      const uint32_t idesc = idesc_bf16_f32(128, 64, 0, 0);
#pragma unroll
      for (int s = 0; s < 8; ++s) {
        const uint32_t koff = (s >> 2) * 16384 + (s & 3) * 32;
        umma_bf16(tmem + kP1TmQK, sdesc_sw128(a_qkw + koff, 16, 1024),
                  sdesc_sw128(a_qkw + 8192 + koff, 16, 1024), idesc, s > 0 ? 1u : 0u);
      }
      umma_commit(bar_mma);
    }
    if (!mbar_wait(bar_mma, 0)) code |= kStatusMmaTimeout;
    tc_fence_after();
    pa_epilogue(tmem + tm_lane + kP1TmQK, row, half, quad, clen, gam, bet, tpzt + 8192, AF);
    tc_fence_before();
    __syncthreads();
    solve_unit_lower(AF, TF, XS, tpzt, bet, eg, tid);
    fence_proxy_async_smem();
    __syncthreads();
    // D_W = [T' ; P] K, with K as the MN-major B operand (64-column blocks 16 KiB apart).
    if (tid == 0) {
      tc_fence_after();
      const uint32_t idesc = idesc_bf16_f32(128, 128, 0, 1);
#pragma unroll
      for (int s = 0; s < 4; ++s)
        umma_bf16(tmem + kP1TmW, sdesc_sw128(a_tpzt + s * 32, 16, 1024),
                  sdesc_sw128(a_qkw + 8192 + s * 2048, 16384, 1024), idesc, s > 0 ? 1u : 0u);
      umma_commit(bar_mma);
    }
    if (row < 64) {
      if (!mbar_wait(bar_mma, 1)) code |= kStatusMmaTimeout;
      tc_fence_after();
      float r[64];
      tmem_ld64(tmem + tm_lane + kP1TmW + 64 * half, r);
      uint8_t* tile = smem + kP1OffQKW + half * 16384;
      st_half_row_bf16(tile, 64 + row, 0, r, -1.0f);   // -W over the consumed K rows
      st_half_row_bf16(tile, 64 + row, 4, r + 32, -1.0f);
    } else {
      scale_q_row(smem + kP1OffQKW + half * 16384, row - 64, eg[row - 64]);
    }
    fence_proxy_async_smem();
    __syncthreads();
    // Tile images out by bulk copies: [e^g Q ; -W], P, T_b, gamma.
    if (tid == 0) {
      uint8_t* rec = sp.records + (static_cast<size_t>(gc) * p.h_v + head) * kRecBytes;
      bulk_store(rec + kRecOffQW, smem + kP1OffQKW, 32768);
      bulk_store(rec + kRecOffP, tpzt + 8192, 8192);
      bulk_store(rec + kRecOffTb, tpzt + 24576, 8192);
      bulk_store(rec + kRecOffGam, gam, 256);
      bulk_commit_and_wait_read();
    }
  }
  if (code) atomicOr(p.status, code);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, kP1TmCols);
}

// ---------------------------------------------------------------- chain kernel
constexpr uint32_t kC2StQW = 0;         // 32 KiB  [e^g Q ; -W]
constexpr uint32_t kC2StP = 32768;      // 8 KiB   P    } stacked [P ; Z] and [Z ; T_b]
constexpr uint32_t kC2StZ = 40960;      // 8 KiB   Z    }
constexpr uint32_t kC2StTb = 49152;     // 8 KiB   T_b  }
constexpr uint32_t kC2StK = 57344;      // 16 KiB  K chunk [c][kd]
constexpr uint32_t kC2StV = 73728;      // 8 KiB   V chunk, this CTA's 64 columns [c][v]
constexpr uint32_t kC2StGam = 81920;    // 256 B   gamma
constexpr uint32_t kC2Stage = 82944;    // 81 KiB per stage
constexpr uint32_t kC2OffSB = 2 * kC2Stage;          // 16 KiB S_s^T bf16 [kd][64 v]
constexpr uint32_t kC2OffVN = kC2OffSB + 16384;      // 8 KiB v_new [c][64 v]
constexpr uint32_t kC2OffVND = kC2OffVN + 8192;      // 8 KiB decayed v_new
constexpr uint32_t kC2OffBar = kC2OffVND + 8192;     // 2 load + 2 UMMA barriers
constexpr uint32_t kC2OffTmemPtr = kC2OffBar + 32;
constexpr uint32_t kC2Smem = kC2OffTmemPtr + 16 + 1024;
constexpr uint32_t kC2TmUO = 0;         // 2 x 64 columns (double-buffered)
constexpr uint32_t kC2TmS4 = 128;       // 64 columns
constexpr uint32_t kC2TmCols = 256;
constexpr uint32_t kC2LoadBytes = 32768 + 8192 + 8192 + 256 + 16384 + 8192;

__global__ void __launch_bounds__(kPrefillThreads, 1)
    gdn_prefill_chain_kernel(const __grid_constant__ CUtensorMap tm_k,
                             const __grid_constant__ CUtensorMap tm_v, const SplitParams sp) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const PrefillParams& p = sp.base;
  const int head = blockIdx.x >> 1, vs = blockIdx.x & 1, seq = blockIdx.y;
  const int hq = head / (p.h_v / p.h_qk);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quad = warp & 3, half = warp >> 2, row = quad * 32 + lane;
  const int gc0 = sp.seq_off[seq];
  const int nch = sp.seq_off[seq + 1] - gc0;
  // this CTA's slice: state rows v in [64 vs, 64 vs + 64)
  const size_t sbase = (static_cast<size_t>(seq) * p.h_v + head) * kHeadDim * kHeadDim +
                       static_cast<size_t>(64 * vs) * kHeadDim;

  if (nch <= 0) {   // ref kernel_prefill.cu:61-66: the state passes through unchanged
    float4* dst = reinterpret_cast<float4*>(p.new_state + sbase);
    const float4* src = p.state ? reinterpret_cast<const float4*>(p.state + sbase) : nullptr;
    for (int i = tid; i < 64 * kHeadDim / 4; i += kPrefillThreads)
      dst[i] = src ? src[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    return;
  }

  uint64_t* bar_ld = reinterpret_cast<uint64_t*>(smem + kC2OffBar);   // [2]
  uint64_t* bar_mma = bar_ld + 2;
  uint64_t* bar_mma2 = bar_ld + 3;
  uint32_t* tmem_ptr = reinterpret_cast<uint32_t*>(smem + kC2OffTmemPtr);

  auto issue_loads = [&](int ci) {   // stage ci & 1 <- chunk ci of this sequence
    const int st = ci & 1;
    uint8_t* stage = smem + st * kC2Stage;
    const int gc = gc0 + ci;
    const ChunkInfo info = sp.table[gc];
    const uint8_t* rec = sp.records + (static_cast<size_t>(gc) * p.h_v + head) * kRecBytes;
    mbar_arrive_expect_tx(bar_ld + st, kC2LoadBytes);
    bulk_load(stage + kC2StQW, rec + kRecOffQW, 32768, bar_ld + st);
    bulk_load(stage + kC2StP, rec + kRecOffP, 8192, bar_ld + st);
    bulk_load(stage + kC2StTb, rec + kRecOffTb, 8192, bar_ld + st);
    bulk_load(stage + kC2StGam, rec + kRecOffGam, 256, bar_ld + st);
    const int t0 = static_cast<int>(info.cstart);
    tma_load_3d(stage + kC2StK, &tm_k, bar_ld + st, 0, hq, t0);
    tma_load_3d(stage + kC2StK + 8192, &tm_k, bar_ld + st, 64, hq, t0);
    tma_load_3d(stage + kC2StV, &tm_v, bar_ld + st, 64 * vs, head, t0);
  };

  if (warp == 0) {
    tmem_alloc(tmem_ptr, kC2TmCols);
    tmem_relinquish();
  }
  if (tid == 32) {
    for (int i = 0; i < 4; ++i) mbar_init(bar_ld + i, 1);
    fence_mbarrier_init();
    prefetch_tmap(&tm_k);
    prefetch_tmap(&tm_v);
  }
  for (int i = tid; i < 512; i += kPrefillThreads) {   // Z blocks of both stages
    reinterpret_cast<uint4*>(smem + kC2StZ)[i] = make_uint4(0, 0, 0, 0);
    reinterpret_cast<uint4*>(smem + kC2Stage + kC2StZ)[i] = make_uint4(0, 0, 0, 0);
  }
  __syncthreads();
  if (tid == 0) {
    issue_loads(0);
    if (nch > 1) issue_loads(1);
  }
  // Thread (k = row, half) holds S_s^T[k][32 half + j] = S[64 vs + 32 half + j][k].
  float sreg[32];
#pragma unroll
  for (int j = 0; j < 32; ++j)
    sreg[j] = p.state ? p.state[sbase + static_cast<size_t>(32 * half + j) * kHeadDim + row] : 0.f;
  st_half_row_bf16(smem + kC2OffSB, row, 4 * half, sreg, 1.0f);
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_ptr;
  const uint32_t tm_lane = static_cast<uint32_t>(quad * 32) << 16;
  const uint32_t a_sb = smem_u32(smem + kC2OffSB);
  const uint32_t a_vn = smem_u32(smem + kC2OffVN);
  const uint32_t a_vnd = smem_u32(smem + kC2OffVND);

  bool failed = false;
  unsigned int fail_code = 0;
  auto wait = [&](uint64_t* bar, uint32_t parity, unsigned int code) {
    if (!mbar_wait(bar, parity)) {
      failed = true;
      fail_code |= code;
    }
  };
  // bar_mma completes twice per chunk (parity 0: U + S^T products, parity 1:
  // state increment); bar_mma2 once per chunk (the P v_new product, parity =
  // chunk & 1); bar_ld[stage] once per use of the stage (parity = (chunk >> 1) & 1).
  auto output_rows = [&](int cj) {   // rows 0-63 of D_UO of chunk cj -> output
    wait(bar_mma2, cj & 1, kStatusMmaTimeout);
    tc_fence_after();
    const ChunkInfo info = sp.table[gc0 + cj];
    float r[32];
    tmem_ld32(tmem + kC2TmUO + 64 * (cj & 1) + tm_lane + 32 * half, r);
    tmem_wait_ld();
    if (row < info.clen) {
      __nv_bfloat16* orow = p.out + (static_cast<size_t>(info.cstart + row) * p.h_v + head) *
                                        kHeadDim + 64 * vs + 32 * half;
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        uint4 u;
        u.x = pack_bf16x2(p.scale * r[8 * cc + 0], p.scale * r[8 * cc + 1]);
        u.y = pack_bf16x2(p.scale * r[8 * cc + 2], p.scale * r[8 * cc + 3]);
        u.z = pack_bf16x2(p.scale * r[8 * cc + 4], p.scale * r[8 * cc + 5]);
        u.w = pack_bf16x2(p.scale * r[8 * cc + 6], p.scale * r[8 * cc + 7]);
        *reinterpret_cast<uint4*>(orow + 8 * cc) = u;
      }
    }
  };
  auto stage_ready = [&](int cj) {   // wait for chunk cj's tiles; clear rows past its end
    const int sj = cj & 1;
    wait(bar_ld + sj, (cj >> 1) & 1, kStatusTmaTimeout);
    const int clen = sp.table[gc0 + cj].clen;
    if (clen < kChunk) {
      uint8_t* stage = smem + sj * kC2Stage;
      const int nrow = kChunk - clen;
      for (int e = tid; e < 3 * nrow * 8; e += kPrefillThreads) {
        const int reg = e / (nrow * 8);
        const int r = clen + (e / 8) % nrow;
        const uint32_t base = reg < 2 ? kC2StK + reg * 8192 : kC2StV;
        *reinterpret_cast<uint4*>(stage + base + sw128_off(r, e & 7)) = make_uint4(0, 0, 0, 0);
      }
      fence_proxy_async_smem();
    }
  };

  stage_ready(0);
  __syncthreads();
  for (int ci = 0; ci < nch; ++ci) {
    const int st = ci & 1;
    uint8_t* stage = smem + st * kC2Stage;
    const uint32_t a_stage = smem_u32(stage);
    const int clen = sp.table[gc0 + ci].clen;
    const uint32_t d_uo = tmem + kC2TmUO + 64 * st;
    const float* gam = reinterpret_cast<const float*>(stage + kC2StGam);

    // D_UO = [Z ; T_b] V_s + [e^g Q ; -W] S_s^T
    if (tid == 0) {
      tc_fence_after();
      const uint32_t idesc = idesc_bf16_f32(128, 64, 0, 1);
#pragma unroll
      for (int s = 0; s < 4; ++s)
        umma_bf16(d_uo, sdesc_sw128(a_stage + kC2StZ + s * 32, 16, 1024),
                  sdesc_sw128(a_stage + kC2StV + s * 2048, 8192, 1024), idesc, s > 0 ? 1u : 0u);
#pragma unroll
      for (int s = 0; s < 8; ++s)
        umma_bf16(d_uo, sdesc_sw128(a_stage + kC2StQW + (s >> 2) * 16384 + (s & 3) * 32, 16, 1024),
                  sdesc_sw128(a_sb + s * 2048, 16384, 1024), idesc, 1u);
      umma_commit(bar_mma);
    }
    // the previous chunk's output rows, while the tensor core works on this one
    if (row < 64 && ci > 0) output_rows(ci - 1);
    wait(bar_mma, 0, kStatusMmaTimeout);
    tc_fence_after();

    const float gam_last = gam[clen - 1];
    if (row >= 64) {   // v_new rows
      const int c = row - 64;
      const float dec = (c < clen) ? __expf(gam_last - gam[c]) : 0.f;
      const float keep = (c < clen) ? 1.f : 0.f;
      float r[32];
      tmem_ld32(d_uo + tm_lane + 32 * half, r);
      tmem_wait_ld();
      st_half_row_bf16(smem + kC2OffVN, c, 4 * half, r, keep);
      st_half_row_bf16(smem + kC2OffVND, c, 4 * half, r, dec);
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();

    // D_S4 = K^T (v_new e^{gamma_last - gamma});  D_UO += [P ; Z] v_new
    if (tid == 0) {
      tc_fence_after();
      const uint32_t idesc_s = idesc_bf16_f32(128, 64, 1, 1);
      const uint32_t idesc_o = idesc_bf16_f32(128, 64, 0, 1);
#pragma unroll
      for (int s = 0; s < 4; ++s)
        umma_bf16(tmem + kC2TmS4, sdesc_sw128(a_stage + kC2StK + s * 2048, 8192, 1024),
                  sdesc_sw128(a_vnd + s * 2048, 8192, 1024), idesc_s, s > 0 ? 1u : 0u);
      umma_commit(bar_mma);
#pragma unroll
      for (int s = 0; s < 4; ++s)
        umma_bf16(d_uo, sdesc_sw128(a_stage + kC2StP + s * 32, 16, 1024),
                  sdesc_sw128(a_vn + s * 2048, 8192, 1024), idesc_o, 1u);
      umma_commit(bar_mma2);
    }
    wait(bar_mma, 1, kStatusMmaTimeout);
    tc_fence_after();
    {   // S_s^T = e^{gamma_last} S_s^T + D_S4
      const float decay = __expf(gam_last);
      float r[32];
      tmem_ld32(tmem + tm_lane + kC2TmS4 + 32 * half, r);
      tmem_wait_ld();
#pragma unroll
      for (int j = 0; j < 32; ++j) sreg[j] = fmaf(decay, sreg[j], r[j]);
      st_half_row_bf16(smem + kC2OffSB, row, 4 * half, sreg, 1.0f);
    }
    if (tid == 0 && ci + 2 < nch) {
      // stage `st` is free once the P v_new product (its last reader) is done
      wait(bar_mma2, ci & 1, kStatusMmaTimeout);
      issue_loads(ci + 2);
    }
    if (ci + 1 < nch) stage_ready(ci + 1);
    fence_proxy_async_smem();
    tc_fence_before();
    if (__syncthreads_or(failed)) break;
  }
  bool any_fail = __syncthreads_or(failed);
  if (!any_fail && row < 64) output_rows(nch - 1);
  any_fail = __syncthreads_or(failed);
  if (any_fail) {
    if (failed) atomicOr(p.status, fail_code);
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      p.new_state[sbase + static_cast<size_t>(32 * half + j) * kHeadDim + row] = sreg[j];
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, kC2TmCols);
}

}  // namespace gdn
