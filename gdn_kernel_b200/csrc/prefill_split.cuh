// Two-stage chunked prefill: the S-independent work of every (chunk, v-head)
// runs fully parallel in one kernel, and the sequential state recurrence runs
// in a second kernel that only does the S-dependent products.
//
//   gdn_chunk_table_kernel   cu_seqlens -> per-sequence chunk offsets and a flat
//                            table of (sequence, chunk start, chunk length).
//   gdn_prefill_prep_kernel  one CTA per (chunk, v-head), two CTAs per SM:
//                            gates, D_QK = [Q;K]K^T, P and A, the triangular
//                            inverse (T' = T diag(beta e^gamma), T_b = T diag(beta)),
//                            D_X = P [T' | T_b], D_W = [T' ; P T'] K.  It folds
//                            the output's intra-chunk part into two S-free tiles,
//                              Q' = e^gamma Q - P W      P' = P T_b
//                            (O = Q' S^T + P' V is e^g Q S^T + P v_new with
//                            v_new = T_b V - W S^T), and stores the bf16 operand
//                            tiles exactly as they sit in shared memory
//                            (128B-swizzled "tile images"): [Q' ; -W] (32 KiB),
//                            P' (8 KiB), T_b (8 KiB), gamma.
//   gdn_prefill_chain_kernel one CTA per (sequence, v-head, 64-column V slice),
//                            warp-specialised; per chunk
//                              D_UO  = [P' ; T_b] V_s + [Q' ; -W] S_s^T
//                                      (rows 0-63 output, rows 64-127 v_new)
//                              D_S4  = K^T (v_new e^{gamma_last-gamma})
//                              S_s^T = e^{gamma_last} S_s^T + D_S4
//                            with only the S-dependent steps serial per chunk.
//
// Both paths compute the same recurrence with bf16 operands and fp32
// accumulation and agree with the oracle to the same stated tolerance; the
// folded tiles Q' and P' round once more to bf16 than the single-kernel path.
// The workspace holds the tables and one 49 KiB record per (chunk, v-head);
// it is caller-provided (gdn_b200_prefill_workspace_size), 256-byte aligned
// (records sit at 1 KiB multiples from its start), or the library's static
// record ring, which holds the records of two windows of chunks at a time.
#pragma once

#include "prefill_kernel.cuh"

namespace gdn {

struct ChunkInfo {
  int seq;
  int clen;           // 0 marks a table slot past the last chunk
  long long cstart;
};

// Record of one (chunk, v-head) in the workspace.
constexpr uint32_t kRecOffQW = 0;          // [Q' ; -W] tile image, 32 KiB
constexpr uint32_t kRecOffP = 32768;       // P' = P T_b tile image, 8 KiB (T_b follows)
constexpr uint32_t kRecOffTb = 40960;      // T_b tile image, 8 KiB
constexpr uint32_t kRecOffGam = 49152;     // gamma[64], 256 B
constexpr uint32_t kRecBytes = 50176;      // 49 KiB (keeps records 1 KiB aligned)

struct SplitLayout {
  size_t off_header, off_seq, off_order, off_table, off_win, off_rec, total;
  long long max_chunks;
};

// Tables plus `rec_rows` rows of H_v records (rec_rows < 0: one row per chunk
// of the table, every record of the call resident at once).  `windows`: room
// for the per-window sequence ranges of an interleaved table.
__host__ __device__ inline SplitLayout split_layout(long long num_seqs, long long total_tokens,
                                                    int h_v, long long rec_rows = -1,
                                                    bool windows = false) {
  SplitLayout L;
  L.max_chunks = (total_tokens + kChunk - 1) / kChunk + num_seqs;
  auto up = [](size_t x, size_t a) { return (x + a - 1) / a * a; };
  L.off_header = 0;
  L.off_seq = 256;
  L.off_order = up(L.off_seq + static_cast<size_t>(num_seqs + 1) * 4, 256);
  L.off_table = up(L.off_order + static_cast<size_t>(num_seqs) * 4, 1024);
  L.off_win = up(L.off_table + static_cast<size_t>(L.max_chunks) * sizeof(ChunkInfo), 256);
  L.off_rec = up(L.off_win + (windows ? static_cast<size_t>(L.max_chunks) * 2 * sizeof(int) : 0),
                 1024);
  const long long rows = rec_rows < 0 ? L.max_chunks : rec_rows;
  L.total = L.off_rec + static_cast<size_t>(rows) * h_v * kRecBytes;
  return L;
}

struct SplitParams {
  PrefillParams base;
  int zero_v;             // chain kernel: V is all zero (no V tiles, no M1); out may be null
  int* header;            // [0] = total chunks
  int* seq_off;           // [N + 1] first chunk of each sequence
  int* order;             // [N] sequence of each chain CTA row (grid row y runs order[y])
  ChunkInfo* table;       // [max_chunks]
  uint8_t* records;       // [ring_rows][H_v] x kRecBytes
  int num_seqs;
  int max_chunks;
  // Records of table chunk g live in row g % ring_rows (ring_rows = max_chunks:
  // one row per chunk; fewer: a ring that consecutive windows reuse).
  int ring_rows;
  // Prep kernel: launched to follow the chunk-table kernel (programmatic
  // serialization), so it waits for that grid before reading the table.
  int wait_table;
  // Chunk window [c_lo, c_hi) of table (global) chunk indices: the prep kernel
  // does the items of those chunks, the chain kernel those chunks of every
  // sequence.  The whole call is [0, INT_MAX).  A sequence whose first chunk
  // lies before the window continues from new_state, where the previous
  // window left it.
  int c_lo, c_hi;
  // Table order.  group = 1: sequence-major (sequence i's chunks at
  // seq_off[i] ..).  group > 1: the chunks of each group of `group`
  // consecutive sequences occupy the same span as in sequence-major order but
  // are interleaved in rounds: round r holds chunks [r block, (r + 1) block)
  // of every member, member by member.  A window then holds chunks of all the
  // members of a group, each a consecutive run of its own chunks.
  int group, block;
  // Windows of an interleaved table: `window` chunks each (0: none).  The
  // chunk-table kernel writes, per window w, the range [win_seq[2 w],
  // win_seq[2 w + 1]) of sequences whose groups overlap it.  With scan set,
  // CTA row blockIdx.y of the chain kernel runs the candidates of window
  // c_lo / window: the range's first sequence + blockIdx.y, + gridDim.y, ...;
  // otherwise CTA row y runs sequence y.
  int window;
  int scan;
  int* win_seq;           // [2 x ceil(max_chunks / window)]
  // Failure-detection self-test of the chain kernel: a wait limit (0: the
  // default kWaitLimitNs), and a chunk from which the producer issues no more
  // loads (-1: none), so that a wait nothing will satisfy runs out.
  unsigned long long wait_limit_ns;
  int withhold_from;
};

constexpr int kMaxGroup = 16;

__device__ __forceinline__ uint8_t* record_at(const SplitParams& sp, int g, int head) {
  // (no division unless the rows wrap: this sits on the producer's path)
  const int row = g < sp.ring_rows ? g : g % sp.ring_rows;
  return sp.records + (static_cast<size_t>(row) * sp.base.h_v + head) * kRecBytes;
}

// A sequence's group: the table span of the group and the members' chunk
// counts (read from seq_off as needed; no per-thread array).
struct GroupView {
  int g0, base, members, rank, n;   // first member, span start, members, rank of this one, its chunks
};

__device__ inline GroupView group_view(const SplitParams& sp, int seq) {
  GroupView g;
  g.g0 = sp.group > 1 ? seq - seq % sp.group : seq;
  g.members = sp.group > 1 ? min(sp.group, sp.num_seqs - g.g0) : 1;
  g.rank = seq - g.g0;
  g.base = sp.seq_off[g.g0];
  g.n = sp.seq_off[seq + 1] - sp.seq_off[seq];
  return g;
}

// Table position of chunk j of the sequence of `g` (increasing in j).
__device__ inline int chunk_pos(const SplitParams& sp, const GroupView& g, int j) {
  if (sp.group <= 1) return g.base + j;
  const int rb = (j / sp.block) * sp.block;          // first chunk of j's round
  int pos = g.base + (j - rb);
  for (int m = 0; m < g.members; ++m) {
    const int nm = sp.seq_off[g.g0 + m + 1] - sp.seq_off[g.g0 + m];
    pos += min(nm, rb);                                          // the rounds before
    if (m < g.rank) pos += min(sp.block, max(0, nm - rb));      // earlier members, this round
  }
  return pos;
}

// Programmatic dependent launch.  launch_dependents lets the grid launched
// after this one with programmatic stream serialization start once every CTA
// of this grid has issued it (or exited); wait blocks until the grid this one
// was launched after has completed and its memory is visible.  Both do nothing
// for a grid launched without that attribute / without such a dependent.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// ---------------------------------------------------------------- chunk table
constexpr int kTableThreads = 1024;
constexpr int kOrderMax = 512;   // longest-first chain rows for at most this many sequences

// Token range [s0, s1) of sequence i, or an empty range (and the bad-seqlens
// status bit) when the pair is outside 0 <= s0 <= s1 <= total_tokens.
__device__ __forceinline__ void seq_range(const PrefillParams& p, int i, long long& s0,
                                          long long& s1) {
  s0 = load_cu(p, i);
  s1 = load_cu(p, i + 1);
  if (s0 < 0 || s1 < s0 || s1 > p.total_tokens) {
    atomicOr(p.status, kStatusBadSeqlens);   // treated as an empty sequence
    s0 = s1 = 0;
  }
}

// Two passes over the sequences.  Pass 1 scans the per-sequence chunk counts
// into seq_off.  Valid cu_seqlens (non-decreasing, within [0, total_tokens])
// describe disjoint sequences, so the total is at most ceil(T / 64) + N =
// max_chunks, the table's capacity.  Entries that are each in range but not
// ordered can describe overlapping sequences whose chunks exceed it; then the
// status bit is set and every sequence is treated as empty, so no kernel ever
// indexes past max_chunks.  Pass 2 writes the table.
__global__ void __launch_bounds__(kTableThreads) gdn_chunk_table_kernel(SplitParams sp) {
  __shared__ long long warp_sums[32];
  __shared__ long long carry_s;
  // The prep grid after this one may start its setup now (it waits for this
  // grid's completion before it reads the table).
  pdl_launch_dependents();
  const PrefillParams& p = sp.base;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) carry_s = 0;
  __syncthreads();
  for (int base = 0; base < sp.num_seqs; base += kTableThreads) {
    const int i = base + tid;
    int n = 0;
    if (i < sp.num_seqs) {
      long long s0, s1;
      seq_range(p, i, s0, s1);
      n = static_cast<int>((s1 - s0 + kChunk - 1) / kChunk);
    }
    long long x = n;   // inclusive warp scan
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const long long y = __shfl_up_sync(0xffffffffu, x, off);
      if (lane >= off) x += y;
    }
    if (lane == 31) warp_sums[warp] = x;
    __syncthreads();
    if (warp == 0) {
      long long w = warp_sums[lane];
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const long long y = __shfl_up_sync(0xffffffffu, w, off);
        if (lane >= off) w += y;
      }
      warp_sums[lane] = w;   // inclusive over warps
    }
    __syncthreads();
    const long long excl = carry_s + (warp > 0 ? warp_sums[warp - 1] : 0) + x - n;
    if (i < sp.num_seqs) sp.seq_off[i] = static_cast<int>(min(excl, static_cast<long long>(sp.max_chunks)));
    __syncthreads();
    if (tid == kTableThreads - 1) carry_s = excl + n;
    __syncthreads();
  }
  const bool overflow = carry_s > sp.max_chunks;
  const int total = overflow ? 0 : static_cast<int>(carry_s);
  if (tid == 0) {
    if (overflow) atomicOr(p.status, kStatusBadSeqlens);
    sp.seq_off[sp.num_seqs] = total;
    sp.header[0] = total;
  }
  __syncthreads();   // pass 2 reads the chunk counts of a sequence's whole group
  if (!overflow && sp.group <= 1) {
    // Sequence-major table: every thread fills table positions directly (the
    // owner of position c is the last sequence whose first chunk is <= c), so a
    // long sequence's entries are not written by one thread.
    for (int c = tid; c < total; c += kTableThreads) {
      int lo = 0, hi = sp.num_seqs - 1;
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (sp.seq_off[mid] <= c) lo = mid;
        else hi = mid - 1;
      }
      long long s0, s1;
      seq_range(p, lo, s0, s1);
      ChunkInfo e;
      e.seq = lo;
      e.cstart = s0 + static_cast<long long>(c - sp.seq_off[lo]) * kChunk;
      e.clen = static_cast<int>(min(static_cast<long long>(kChunk), s1 - e.cstart));
      sp.table[c] = e;
    }
  }
  for (int i = tid; i < sp.num_seqs; i += kTableThreads) {
    if (overflow) {   // overlapping sequences: all are treated as empty
      sp.seq_off[i] = 0;
      continue;
    }
    if (sp.group <= 1) continue;   // written above
    long long s0, s1;
    seq_range(p, i, s0, s1);
    const GroupView g = group_view(sp, i);
    const int n = static_cast<int>((s1 - s0 + kChunk - 1) / kChunk);
    const int run = sp.group > 1 ? sp.block : max(n, 1);   // chunks at consecutive positions
    for (int k0 = 0; k0 < n; k0 += run) {
      const int pos = chunk_pos(sp, g, k0);
      for (int k = k0; k < min(n, k0 + run); ++k) {
        ChunkInfo c;
        c.seq = i;
        c.cstart = s0 + static_cast<long long>(k) * kChunk;
        c.clen = static_cast<int>(min(static_cast<long long>(kChunk), s1 - c.cstart));
        sp.table[pos + (k - k0)] = c;
      }
    }
  }
  // The chain kernel's CTA rows: up to kOrderMax sequences of a sequence-major
  // table longest first (ties: lower index), so that its first wave takes the
  // long chains and the short ones fill in behind them; otherwise in index
  // order.  Rank by counting, on the chunk counts staged in shared memory.
  {
    __shared__ int counts[kOrderMax];
    const bool sort = !overflow && sp.group <= 1 && sp.num_seqs > 1 && sp.num_seqs <= kOrderMax;
    if (sort) {
      for (int i = tid; i < sp.num_seqs; i += kTableThreads)
        counts[i] = sp.seq_off[i + 1] - sp.seq_off[i];
      __syncthreads();
    }
    for (int i = tid; i < sp.num_seqs; i += kTableThreads) {
      int rank = i;
      if (sort) {
        const int ni = counts[i];
        rank = 0;
        for (int j = 0; j < sp.num_seqs; ++j) rank += counts[j] > ni || (counts[j] == ni && j < i);
      }
      sp.order[rank] = i;
    }
  }
  // Windows of an interleaved table: the sequences of the groups that
  // overlap each window (windows past the table's end get an empty range).
  if (sp.window > 0) {
    const int groups = (sp.num_seqs + sp.group - 1) / sp.group;
    auto group_of = [&](int c) {   // the last group whose span starts at or before c
      int lo = 0, hi = groups - 1;
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (sp.seq_off[mid * sp.group] <= c) lo = mid;
        else hi = mid - 1;
      }
      return lo;
    };
    const int nwin = (sp.max_chunks + sp.window - 1) / sp.window;
    for (int w = tid; w < nwin; w += kTableThreads) {
      const long long c0 = static_cast<long long>(w) * sp.window;
      int s_lo = 0, s_hi = 0;
      if (c0 < total) {
        const int c1 = static_cast<int>(min(c0 + sp.window, static_cast<long long>(total))) - 1;
        s_lo = group_of(static_cast<int>(c0)) * sp.group;
        s_hi = min(sp.num_seqs, (group_of(c1) + 1) * sp.group);
      }
      sp.win_seq[2 * w] = s_lo;
      sp.win_seq[2 * w + 1] = s_hi;
    }
  }
  // Table slots past the last chunk get clen = 0: the prep kernel's CTAs for
  // them read one entry and exit.
  for (int i = total + tid; i < sp.max_chunks; i += kTableThreads) {
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
// Persistent: two CTAs per SM walk the (chunk, v-head) items in order (item =
// chunk * H_v + head, so consecutive items share Q and K).  Two 35 KiB regions
// take turns: the current item's [Q;K] tile lives in one while its fp32 A / T
// scratch of the triangular solve lives in the other; once the solve is done
// that scratch is dead, and the next item's Q/K copy lands there while this
// item finishes its products and stores.  So the per-item path carries no copy
// latency, no TMEM allocation and no store drain.
constexpr uint32_t kP1Region = 35840;                   // 35 KiB: [Q;K] tile or A + T scratch
constexpr uint32_t kP1OffR0 = 0;
constexpr uint32_t kP1OffTPZT = kP1Region;             // 32 KiB T' | P, then P T' | P' | T_b
constexpr uint32_t kP1OffR1 = kP1OffTPZT + 32768;
constexpr uint32_t kP1TbOff = 24576;                   // T_b within TPZT
constexpr uint32_t kP1OffTFinR = 64 * kLdA * 4;        // T after A within a scratch region
constexpr uint32_t kP1OffXS = kP1OffR1 + kP1Region;
constexpr uint32_t kP1OffGate = kP1OffXS + 32 * 40 * 4;   // 2 gate buffers (gate_finish)
constexpr uint32_t kP1OffBar = kP1OffGate + 2 * kGateFloats * 4;   // TMA [2], QK, X, W
constexpr uint32_t kP1OffTmemPtr = kP1OffBar + 48;
constexpr uint32_t kP1Smem = kP1OffTmemPtr + 16 + 1024;
constexpr uint32_t kP1TmQK = 0;       // 64 columns
constexpr uint32_t kP1TmX = 0;        // 128 columns (D_QK is consumed by then)
constexpr uint32_t kP1TmW = 128;      // 128 columns
constexpr uint32_t kP1TmCols = 256;
static_assert(2 * kP1OffTFinR <= kP1Region, "A and T scratch must fit a region");
constexpr int kP1StoreTid = kPrefillThreads - 32;       // lane 0 of the last warp: record stores
constexpr int kP1BarPT = 1;    // named barrier: P T' tile written (warps 0-1)
constexpr int kP1BarRec = 2;   // named barrier: an item's record tiles complete (store warp waits)
static_assert(kP1Smem + 1024 <= 232448 / 2, "two prep CTAs must fit an SM");

__global__ void __launch_bounds__(kPrefillThreads, 2)
    gdn_prefill_prep_kernel(const __grid_constant__ CUtensorMap tm_q,
                            const __grid_constant__ CUtensorMap tm_k, const SplitParams sp) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const PrefillParams& p = sp.base;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quad = warp & 3, half = warp >> 2, row = quad * 32 + lane;

  // One mbarrier per product, each completing once per item (phase parity =
  // item parity j & 1).  Warps wait on them without a CTA-wide barrier in
  // between, so a shared barrier could be a whole phase ahead of a slow warp
  // and alias its parity; with one per product, the item's first CTA-wide
  // barrier keeps every warp within one phase.
  uint64_t* bar_tma = reinterpret_cast<uint64_t*>(smem + kP1OffBar);   // [2]
  uint64_t* bar_qk = bar_tma + 2;
  uint64_t* bar_x = bar_tma + 3;
  uint64_t* bar_w = bar_tma + 4;
  uint32_t* tmem_ptr = reinterpret_cast<uint32_t*>(smem + kP1OffTmemPtr);
  float* XS = reinterpret_cast<float*>(smem + kP1OffXS);
  uint8_t* tpzt = smem + kP1OffTPZT;
  auto region = [&](int r) { return smem + (r ? kP1OffR1 : kP1OffR0); };
  auto gates = [&](int r) {
    return reinterpret_cast<float*>(smem + kP1OffGate + kGateFloats * 4 * r);
  };

  // The chain grid launched after this one (one-sequence pieces) may be
  // launched now; its CTAs wait for SMs and then for this grid's completion.
  pdl_launch_dependents();
  if (warp == 0) {
    tmem_alloc(tmem_ptr, kP1TmCols);
    tmem_relinquish();
  }
  if (tid == 32) {
    mbar_init(bar_tma, 1);
    mbar_init(bar_tma + 1, 1);
    mbar_init(bar_qk, 1);
    mbar_init(bar_x, 1);
    mbar_init(bar_w, 1);
    fence_mbarrier_init();
    prefetch_tmap(&tm_q);
    prefetch_tmap(&tm_k);
  }
  // The solve never writes the upper-right 32x32 blocks of the T' and T_b
  // tiles (rows 0-31, 16-byte chunks 4-7): they hold zeros for every item.
  {
    const int r = tid >> 3, c = 4 + ((tid >> 1) & 3), t = tid & 1;
    *reinterpret_cast<uint4*>(tpzt + 24576 * t + sw128_off(r, c)) = make_uint4(0, 0, 0, 0);
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_ptr;
  const uint32_t tm_lane = static_cast<uint32_t>(quad * 32) << 16;
  const uint32_t a_tpzt = smem_u32(tpzt);
  // The first prep of a call is launched to follow the chunk-table kernel and
  // may start before the table is complete: the setup above reads nothing the
  // table kernel writes, and the wait here precedes every table read.
  if (sp.wait_table) pdl_wait();
  const int n_chunks = min(sp.header[0], sp.c_hi);

  // Items are (chunk, v-head) pairs in chunk-major order; a CTA steps through
  // them gridDim.x at a time, i.e. by (dc chunks, dh heads), without dividing.
  struct Item {
    int c, h;
  };
  const int dc = static_cast<int>(gridDim.x) / p.h_v, dh = static_cast<int>(gridDim.x) % p.h_v;
  auto advance = [&](Item x) {
    x.c += dc;
    x.h += dh;
    if (x.h >= p.h_v) {
      x.h -= p.h_v;
      ++x.c;
    }
    return x;
  };
  auto table_at = [&](const Item& x) {
    return x.c < n_chunks ? sp.table[x.c] : ChunkInfo{-1, 0, 0};
  };
  // An item's Q/K tiles into region r (the store thread, off warp 0's path).
  auto issue_tiles = [&](const Item& x, const ChunkInfo& info, int r) {
    if (tid == kP1StoreTid) {
      const int hq = x.h / (p.h_v / p.h_qk);
      const int t0 = static_cast<int>(info.cstart);
      mbar_arrive_expect_tx(bar_tma + r, 4 * kTileBytes);
#pragma unroll
      for (int kb = 0; kb < 2; ++kb) {
        tma_load_3d(region(r) + kb * 16384, &tm_q, bar_tma + r, kb * 64, hq, t0);
        tma_load_3d(region(r) + kb * 16384 + 8192, &tm_k, bar_tma + r, kb * 64, hq, t0);
      }
    }
  };
  // An item's gate inputs into warp 1's registers, issued a whole item before
  // gate_finish needs them (a, b and the head's A_log, dt_bias).
  float g_alog = 0.f, g_dtb = 0.f;
  auto load_gates = [&](const Item& x, const ChunkInfo& info, GateIn& gi) {
    if (warp == 1) {
      gi = gate_inputs(p, info.cstart, info.clen, x.h, lane);
      g_alog = p.A_log[x.h];
      g_dtb = p.dt_bias[x.h];
    }
  };
  auto finish_gates = [&](const GateIn& gi, int r) {
    if (warp == 1) {
      float* g = gates(r);
      gate_finish(gi, -expf(g_alog), g_dtb, lane, g, g + 64, g + 128, g + 192);
    }
  };

  unsigned int code = 0;
  int w_issued = 0;           // W commits so far (the drain's commit follows them)
  bool failed = false;
  int pend_r = -1;            // region whose copy is in flight and not yet waited for
  uint32_t pend_parity = 0;
  Item cur{sp.c_lo + static_cast<int>(blockIdx.x) / p.h_v, static_cast<int>(blockIdx.x) % p.h_v};
  Item nxt = advance(cur);
  ChunkInfo cur_info = table_at(cur);
  ChunkInfo nxt_info = table_at(nxt);
  GateIn gi{};
  if (cur.c < n_chunks) {
    issue_tiles(cur, cur_info, 0);
    pend_r = 0;
    pend_parity = 0;
    load_gates(cur, cur_info, gi);
    finish_gates(gi, 0);
  }
  for (int j = 0; cur.c < n_chunks; ++j) {
    const int r = j & 1;
    const int gc = cur.c, head = cur.h;
    const bool has_nxt = nxt.c < n_chunks;
    const Item nx2 = advance(nxt);
    const ChunkInfo nx2_info = table_at(nx2);   // used an item from now
    if (has_nxt) load_gates(nxt, nxt_info, gi);
    const int clen = cur_info.clen;
    uint8_t* qkw = region(r);
    float* AF = reinterpret_cast<float*>(region(r ^ 1));
    float* TF = reinterpret_cast<float*>(region(r ^ 1) + kP1OffTFinR);
    float* gam = gates(r);
    float* bet = gam + 64;
    float* eg = gam + 128;
    const uint32_t a_qkw = smem_u32(qkw);

    bool ok = mbar_wait(bar_tma + r, (j >> 1) & 1);
    if (ok) pend_r = -1;
    else code |= kStatusTmaTimeout;

    // D_QK = [Q ; K] K^T, with K (rows 64-127 of the stacked tile) as the B
    // operand, issued by warp 0 as soon as the tiles have landed: no CTA-wide
    // barrier first (this item's gates were published by the previous item's
    // last one, and the same warp zeroes the rows past a short chunk's end).
    if (warp == 0) {
      if (ok && clen < kChunk) {
        const int nrow = kChunk - clen;
        for (int e = lane; e < 4 * nrow * 8; e += 32) {
          const int reg = e / (nrow * 8);
          const int rr = clen + (e / 8) % nrow;
          *reinterpret_cast<uint4*>(qkw + (reg >> 1) * 16384 + (reg & 1) * 8192 +
                                    sw128_off(rr, e & 7)) = make_uint4(0, 0, 0, 0);
        }
        fence_proxy_async_smem();
      }
      __syncwarp();
      tc_fence_after();
      if (ok && elect_one()) {
        const uint32_t idesc = idesc_bf16_f32(128, 64, 0, 0);
#pragma unroll
        for (int s = 0; s < 8; ++s) {
          const uint32_t koff = (s >> 2) * 16384 + (s & 3) * 32;
          umma_bf16(tmem + kP1TmQK, sdesc_sw128(a_qkw + koff, 16, 1024),
                    sdesc_sw128(a_qkw + 8192 + koff, 16, 1024), idesc, s > 0 ? 1u : 0u);
        }
        umma_commit(bar_qk);
      }
      __syncwarp();
    }
    // The previous item's records must have been read out of TPZT and the
    // other region (its [Q;K] tile) before the P/A epilogue overwrites them.
    if (tid == kP1StoreTid) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
    if (ok) {
      ok = mbar_wait(bar_qk, j & 1);
      if (!ok) code |= kStatusMmaTimeout;
    }
    // (also the first CTA-wide barrier after a failure in the previous item)
    if (__syncthreads_or(!ok || code != 0)) { failed = true; break; }
    tc_fence_after();
    pa_epilogue(tmem + tm_lane + kP1TmQK, row, half, quad, clen, gam, bet, gam + 192, tpzt + 8192,
                AF);
    // The next item's gates (loaded at the top of this item) into the other
    // buffer, by warp 1, which finishes its share of the epilogue early.  That
    // buffer's previous contents (item j - 1's gamma) left with item j - 1's
    // records, whose read-out the store thread waited for before the barrier
    // above.  At the end of the item this made warp 1 the last warp into the
    // next item's first barrier.
    if (has_nxt) finish_gates(gi, r ^ 1);
    tc_fence_before();
    __syncthreads();
    solve_unit_lower(AF, TF, XS, tpzt, bet, eg, tid);
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    // The solve's scratch is dead: the next item's tiles go there now.
    if (has_nxt) {
      issue_tiles(nxt, nxt_info, r ^ 1);
      pend_r = r ^ 1;
      pend_parity = ((j + 1) >> 1) & 1;
    }
    // D_X = [P ; -] [T' | T_b]: P T' (columns 0-63) and P' = P T_b (64-127).
    // Rows 64-127 of the A operand are scratch; their products are not read.
    // The B operand's two 64-column blocks are the T' and T_b tiles.
    if (warp == 0) {
      tc_fence_after();
      if (elect_one()) {
        const uint32_t idesc = idesc_bf16_f32(128, 128, 0, 1);
#pragma unroll
        for (int s = 0; s < 4; ++s)
          umma_bf16(tmem + kP1TmX, sdesc_sw128(a_tpzt + 8192 + s * 32, 16, 1024),
                    sdesc_sw128(a_tpzt + s * 2048, kP1TbOff, 1024), idesc, s > 0 ? 1u : 0u);
        umma_commit(bar_x);
      }
      __syncwarp();
    }
    if (quad < 2) {   // half 0: P T' over P (A rows 64-127 of D_W); half 1: P' to the scratch rows
      if (!mbar_wait(bar_x, j & 1)) code |= kStatusMmaTimeout;
      tc_fence_after();
      float rr[64];
      tmem_ld64(tmem + tm_lane + kP1TmX + 64 * half, rr);
      st_row_bf16(tpzt + (half == 0 ? 8192 : 16384), row, rr);
    }
    fence_proxy_async_smem();
    // D_W = [T' ; P T'] K, K the MN-major B operand (64-column blocks 16 KiB
    // apart): rows 0-63 W = T'K, rows 64-127 P W.  Its A operand needs P T'
    // from warps 0 and 1 only (P' from warps 4 and 5 leaves with the records).
    if (warp < 2) {
      tc_fence_before();
      named_sync(kP1BarPT, 64);
    }
    if (warp == 0) {
      tc_fence_after();
      if (elect_one()) {
        const uint32_t idesc = idesc_bf16_f32(128, 128, 0, 1);
#pragma unroll
        for (int s = 0; s < 4; ++s)
          umma_bf16(tmem + kP1TmW, sdesc_sw128(a_tpzt + s * 32, 16, 1024),
                    sdesc_sw128(a_qkw + 8192 + s * 2048, 16384, 1024), idesc, s > 0 ? 1u : 0u);
        umma_commit(bar_w);
      }
      __syncwarp();
    }
    ++w_issued;
    ok = mbar_wait(bar_w, j & 1);
    if (!ok) code |= kStatusMmaTimeout;
    tc_fence_after();
    if (ok) {
      float rr[64];
      tmem_ld64(tmem + tm_lane + kP1TmW + 64 * half, rr);
      uint8_t* tile = qkw + half * 16384;
      if (row < 64) {   // -W over the consumed K rows
        st_half_row_bf16(tile, 64 + row, 0, rr, -1.0f);
        st_half_row_bf16(tile, 64 + row, 4, rr + 32, -1.0f);
      } else {          // Q' = e^gamma Q - P W over the Q rows
        qprime_row(tile, row - 64, eg[row - 64], rr);
      }
    }
    fence_proxy_async_smem();
    tc_fence_before();
    // Only the store thread's warp waits for the finished tiles; the others
    // go on to the next item (its first CTA-wide barrier catches failures).
    if (tid >= kP1StoreTid) named_sync(kP1BarRec, kPrefillThreads);
    else named_arrive(kP1BarRec, kPrefillThreads);
    // Tile images out by bulk copies ([Q' ; -W], P', T_b, gamma); drained by
    // the next item (or the end of the kernel) before their sources change.
    // A thread of the last warp issues them, off warp 0's path to the next
    // item's first product.  (Writing the [Q' ; -W] rows straight from
    // registers instead, one row per thread, was slower on B200.)
    if (tid == kP1StoreTid) {
      uint8_t* rec = record_at(sp, gc, head);
      bulk_store(rec + kRecOffQW, qkw, 32768);
      bulk_store(rec + kRecOffP, tpzt + 16384, 8192);
      bulk_store(rec + kRecOffTb, tpzt + kP1TbOff, 8192);
      bulk_store(rec + kRecOffGam, gam, 256);
      asm volatile("cp.async.bulk.commit_group;" ::: "memory");
    }
    cur = nxt;
    cur_info = nxt_info;
    nxt = nx2;
    nxt_info = nx2_info;
  }
  // Everything in flight lands before the CTA's shared memory and TMEM go
  // away: bulk stores (the store thread's groups), and on a failed run the
  // copy still pending and the tensor-core ops (one more bounded wait each).
  if (tid == kP1StoreTid) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
  failed = failed || code != 0;
  if (failed) {
    if (pend_r >= 0) mbar_wait(bar_tma + pend_r, pend_parity);
    if (warp == 0) {
      if (elect_one()) umma_commit(bar_w);
      __syncwarp();
    }
    mbar_wait(bar_w, w_issued & 1);
  }
  if (code) atomicOr(p.status, code);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, kP1TmCols);
  // When this grid was launched to overlap the chain kernel before it (a
  // one-sequence call in pieces), it completes only after that kernel: the
  // next piece's chain, launched after this grid, then starts from a finished
  // state.
  pdl_wait();
}

// ---------------------------------------------------------------- chain kernel
// One CTA per (sequence, v-head, kVS-column V slice), warp-specialised:
//   warps 0-7  state warps: thread (k = row, half) keeps S_s^T[k][kVS/2 half + j]
//              in registers; warps 2,3,6,7 also turn rows 64-127 of D_UO into
//              the decayed v_new tile; warp 0 issues M2 and M3.  The eight
//              hand over to one another through two named barriers only;
//   warps 8-9  output warps: rows 0-63 of D_UO -> bf16 output rows;
//   warp 10    producer: bulk/TMA loads, issued as soon as a stage part frees;
//   warp 11    M1, and rows past a short chunk's end zeroed once its tiles land.
// Per chunk c (stage st = c & 1, D_UO double-buffered in TMEM):
//   M1  D_UO[st]  = [P' ; T_b] V          (warp 11; no S, issued ahead)
//   M2  D_UO[st] += [Q' ; -W] S_s^T       -> rows 0-63 output, 64-127 v_new
//   M3  D_S4      = K^T (v_new e^{gamma_last - gamma})
//   S_s^T = e^{gamma_last} S_s^T + D_S4   (bf16 copy -> M2 of chunk c + 1)
// Only M2 -> v_new -> M3 -> state update is serial from chunk to chunk.
// Shared-memory and TMEM layout of a chain CTA that owns kVS of a head's 128
// V columns (kVS = 64: two CTAs per head; 128: one).  The V, S^T and v_new
// tiles are kVS / 64 blocks of 64 columns, each block 128B-swizzled.
template <int kVS>
struct ChainLayout {
  static constexpr int kVBlocks = kVS / 64;
  static constexpr int kCols = kVS / 2;               // state columns per state thread
  static constexpr uint32_t kStQW = 0;                // 32 KiB [Q' ; -W]  (record)
  static constexpr uint32_t kStPT = 32768;            // 16 KiB [P' ; T_b] (record, adjacent there too)
  static constexpr uint32_t kStK = 49152;             // 16 KiB K chunk [c][kd], two 64-column blocks
  static constexpr uint32_t kStV = 65536;             // V chunk, this CTA's columns [c][v]
  static constexpr uint32_t kStGam = kStV + 8192 * kVBlocks;   // 256 B gamma (record)
  static constexpr uint32_t kStage = (kStGam + 256 + 1023) / 1024 * 1024;
  static constexpr uint32_t kOffSB = 2 * kStage;                  // S_s^T bf16 [kd][v]
  static constexpr uint32_t kOffVND = kOffSB + 16384 * kVBlocks;  // decayed v_new [c][v]
  static constexpr uint32_t kOffBar = kOffVND + 8192 * kVBlocks;
  static constexpr uint32_t kOffTmemPtr = kOffBar + 8 * 19;
  static constexpr uint32_t kOffAbort = kOffTmemPtr + 16;
  static constexpr uint32_t kSmem = kOffAbort + 16 + 1024;
  static constexpr uint32_t kTmUO = 0;                // 2 x kVS columns
  static constexpr uint32_t kTmS4 = 2 * kVS;          // kVS columns
  static constexpr uint32_t kTmCols = kVS == 64 ? 256 : 512;
  static constexpr uint32_t kLoadA = 32768 + 16384 + 8192 * kVBlocks + 256;
  static_assert(kVS == 64 || kVS == 128, "a chain CTA owns 64 or 128 V columns");
  static_assert(kSmem <= 232448, "chain CTA shared memory");
};
constexpr uint32_t kC2LoadB = 16384;
// mbarriers (pairs are per stage / D_UO buffer):
//   LdA, LdB   stage loads landed (record + V; K)
//   M1         M1 done (loader's commit)          UO    M2 done (warp 0's commit)
//   Out        output warps have read D_UO[st]    FreeA / FreeB  stage parts reusable
//   KReady     K landed and short rows zeroed     S     M3 done
//   End, End2  drains of an aborted run (warp 0, warp 11)
enum : int {
  kC2BarLdA = 0, kC2BarLdB = 2, kC2BarM1 = 4, kC2BarUO = 6, kC2BarOut = 8,
  kC2BarFreeA = 10, kC2BarFreeB = 12, kC2BarKReady = 14, kC2BarS = 16, kC2BarEnd = 17,
  kC2BarEnd2 = 18, kC2NumBars = 19
};
static_assert(kC2NumBars == 19, "ChainLayout reserves 19 mbarriers");
constexpr int kC2StateWarps = 8;
constexpr int kC2OutWarps = 2;
constexpr int kC2LoaderWarp = kC2StateWarps + kC2OutWarps;
constexpr int kC2M1Warp = kC2LoaderWarp + 1;
constexpr int kC2Threads = 32 * (kC2M1Warp + 1);

// Named barrier among the state warps (ids 1, 2; 0 is __syncthreads).
__device__ __forceinline__ void state_sync(int id) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(32 * kC2StateWarps) : "memory");
}

// kScan: the window form (CTA rows run a window's candidate sequences in turn);
// otherwise CTA row y runs sequence y once.
template <int kVS, bool kScan>
__global__ void __launch_bounds__(kC2Threads, 1)
    gdn_prefill_chain_kernel(const __grid_constant__ CUtensorMap tm_k,
                             const __grid_constant__ CUtensorMap tm_v, const SplitParams sp) {
  using L = ChainLayout<kVS>;
  constexpr int kCols = L::kCols;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const PrefillParams& p = sp.base;
  const int head = blockIdx.x / (kHeadDim / kVS), vs = blockIdx.x % (kHeadDim / kVS);
  const int hq = head / (p.h_v / p.h_qk);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // A chain grid launched with programmatic serialization after the prep that
  // overlapped the chain before it is resident before that chain ends; it waits
  // here until the prep (and so the chain before it) has completed, which
  // precedes every read of a record or state.  Only then may the next piece's
  // prep start, so it cannot take SMs from this grid's CTAs still arriving.
  // This CTA row's sequence (several sequences: longest first, from the
  // chunk-table kernel, which completed before any prep or chain of the call
  // started, so the load may precede the wait below).
  const int row_seq = !kScan && sp.num_seqs > 1 ? sp.order[blockIdx.y] : static_cast<int>(blockIdx.y);
  pdl_wait();
  pdl_launch_dependents();
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kOffBar);
  uint32_t* tmem_ptr = reinterpret_cast<uint32_t*>(smem + L::kOffTmemPtr);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kOffAbort);
  // TMEM is allocated by the first sequence that has chunks here (after its
  // table lookups, so the allocation overlaps nothing on the critical path)
  // and kept for the CTA's later sequences.
  uint32_t tmem = 0;
  bool have_tmem = false;

  // One sequence's chunks of the window.  Returns false once a wait has run out
  // (the CTA then stops).  Every early return is CTA-uniform.
  auto run_sequence = [&](const int seq) -> bool {
  const GroupView gv = group_view(sp, seq);
  const int seq_n = gv.n;
  // this window's chunks of the sequence: j in [j0, j0 + nch).  Sequence-major
  // tables hold them at gv.base + j; interleaved ones are searched (table
  // positions increase with j).
  auto first_pos_at_or_after = [&](int c) {
    int lo = 0, hi = seq_n;
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;
      if (chunk_pos(sp, gv, mid) >= c) hi = mid;
      else lo = mid + 1;
    }
    return lo;
  };
  int j0, nch;
  if (sp.group <= 1) {
    j0 = min(max(sp.c_lo - gv.base, 0), seq_n);
    nch = min(max(sp.c_hi - gv.base, 0), seq_n) - j0;
  } else {
    j0 = first_pos_at_or_after(sp.c_lo);
    nch = first_pos_at_or_after(sp.c_hi) - j0;
  }
  // this CTA's slice: state rows v in [kVS vs, kVS vs + kVS)
  const size_t sbase = (static_cast<size_t>(seq) * p.h_v + head) * kHeadDim * kHeadDim +
                       static_cast<size_t>(kVS * vs) * kHeadDim;

  if (seq_n == 0) {   // ref kernel_prefill.cu:61-66: the state passes through unchanged
    if (sp.c_lo == 0) {     // (once: in the first window)
      float4* dst = reinterpret_cast<float4*>(p.new_state + sbase);
      const float4* src = p.state ? reinterpret_cast<const float4*>(p.state + sbase) : nullptr;
      for (int i = tid; i < kVS * kHeadDim / 4; i += kC2Threads)
        dst[i] = src ? src[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    return true;
  }
  if (nch <= 0) return true;   // none of this sequence's chunks lies in the window
  const float* init = j0 == 0 ? p.state : p.new_state;
  // Chunks of one sequence are consecutive 64-token windows; only the last
  // may be short.
  const long long cstart0 = sp.table[chunk_pos(sp, gv, j0)].cstart;
  const int clen_last = sp.table[chunk_pos(sp, gv, j0 + nch - 1)].clen;
  auto chunk_len = [&](int c) { return c == nch - 1 ? clen_last : kChunk; };
  // Table position of window chunk c, for the producer, which asks in order:
  // positions run consecutively within a round of sp.block chunks.
  int pos_c = -1, pos_v = 0;
  auto table_pos = [&](int c) {
    if (sp.group <= 1) return gv.base + j0 + c;
    if (pos_c >= 0 && c == pos_c + 1 && (j0 + c) % sp.block != 0) pos_v += 1;
    else pos_v = chunk_pos(sp, gv, j0 + c);
    pos_c = c;
    return pos_v;
  };

  auto load_a = [&](int c) {   // record tiles + V of chunk c -> stage c & 1
    const int st = c & 1;
    uint8_t* stage = smem + st * L::kStage;
    uint64_t* bar = bars + kC2BarLdA + st;
    const uint8_t* rec = record_at(sp, table_pos(c), head);
    mbar_arrive_expect_tx(bar, sp.zero_v ? L::kLoadA - 8192 * L::kVBlocks : L::kLoadA);
    bulk_load(stage + L::kStQW, rec + kRecOffQW, 32768, bar);
    bulk_load(stage + L::kStPT, rec + kRecOffP, 16384, bar);
    bulk_load(stage + L::kStGam, rec + kRecOffGam, 256, bar);
    if (!sp.zero_v) {
#pragma unroll
      for (int b = 0; b < L::kVBlocks; ++b)
        tma_load_3d(stage + L::kStV + 8192 * b, &tm_v, bar, kVS * vs + 64 * b, head,
                    static_cast<int>(cstart0 + 64 * c));
    }
  };
  auto load_b = [&](int c) {   // K of chunk c -> stage c & 1
    const int st = c & 1;
    uint8_t* stage = smem + st * L::kStage;
    uint64_t* bar = bars + kC2BarLdB + st;
    const int t0 = static_cast<int>(cstart0 + 64 * c);
    mbar_arrive_expect_tx(bar, kC2LoadB);
    tma_load_3d(stage + L::kStK, &tm_k, bar, 0, hq, t0);
    tma_load_3d(stage + L::kStK + 8192, &tm_k, bar, 64, hq, t0);
  };

  if (!have_tmem && warp == 0) {
    tmem_alloc(tmem_ptr, L::kTmCols);
    tmem_relinquish();
  }
  // (re)initialised per sequence: every phase of the previous sequence has
  // completed and been waited for before the barrier that ended it
  if (warp == kC2LoaderWarp && lane == 0) {
    if (!have_tmem) *abort_flag = 0;
    for (int i = 0; i < kC2NumBars; ++i)
      mbar_init(bars + i, (i == kC2BarOut || i == kC2BarOut + 1) ? kC2OutWarps : 1);
    fence_mbarrier_init();
    prefetch_tmap(&tm_k);
    prefetch_tmap(&tm_v);
    load_a(0);
    load_b(0);
    if (nch > 1) {
      load_a(1);
      load_b(1);
    }
  }
  float sreg[kCols];
  const int quad = warp & 3, half = (warp >> 2) & 1, row = quad * 32 + lane;
  // This thread's kCols columns of row r of the S^T or v_new tile (64-column
  // blocks `block_bytes` apart): half of one block (kVS = 64) or block `half`.
  auto st_cols_bf16 = [&](uint8_t* tile, uint32_t block_bytes, int r, const float* x, float mul) {
    if constexpr (kVS == 64) {
      st_half_row_bf16(tile, r, 4 * half, x, mul);
    } else {
      st_half_row_bf16(tile + half * block_bytes, r, 0, x, mul);
      st_half_row_bf16(tile + half * block_bytes, r, 4, x + 32, mul);
    }
  };
  if (warp < kC2StateWarps) {
#pragma unroll
    for (int j = 0; j < kCols; ++j)
      sreg[j] = init ? init[sbase + static_cast<size_t>(kCols * half + j) * kHeadDim + row] : 0.f;
    st_cols_bf16(smem + L::kOffSB, 16384, row, sreg, 1.0f);
    fence_proxy_async_smem();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (!have_tmem) {
    tmem = *tmem_ptr;
    have_tmem = true;
  }
  const uint32_t tm_lane = static_cast<uint32_t>(quad * 32) << 16;
  const uint32_t idesc_uo = idesc_bf16_f32(128, kVS, 0, 1);

  // Waits are warp-uniform: every lane polls, and the warp proceeds only if
  // all saw the phase complete (a limit that runs out mid-warp cannot split it).
  const unsigned long long limit_ns = sp.wait_limit_ns ? sp.wait_limit_ns : kWaitLimitNs;
  auto warp_wait = [&](int bar, uint32_t parity, unsigned int code) {
    const int r = mbar_wait_or_abort(bars + bar, parity, abort_flag, limit_ns);
    if (r < 0) atomicOr(p.status, code);
    return __all_sync(0xffffffffu, r == 1);
  };
  // Drain of an aborted run: the tensor-core ops this warp issued land
  // before the CTA's TMEM and shared memory go away.
  auto drain_mma = [&](int bar) {
    if (elect_one()) umma_commit(bars + bar);
    __syncwarp();
    mbar_wait(bars + bar, 0);
  };

  if (warp == kC2LoaderWarp) {
    // ------------------------------------------------ producer warp
    // Stage parts are refilled as soon as chunk c - 2 releases them (its M1,
    // M2 and gamma reads for part A, its M3 for part B).
    int issued = nch > 1 ? 2 : 1;
    bool ok = true;
    for (int c = 2; c < nch; ++c) {
      // (self-test: no more loads; every issued one is consumed before the
      // consumers' first wait on a withheld stage)
      if (sp.withhold_from >= 2 && c >= sp.withhold_from) break;
      const int st = c & 1;
      if (!(ok = warp_wait(kC2BarFreeA + st, ((c - 2) >> 1) & 1, kStatusMmaTimeout))) break;
      if (elect_one()) load_a(c);
      __syncwarp();
      if (!(ok = warp_wait(kC2BarFreeB + st, ((c - 2) >> 1) & 1, kStatusMmaTimeout))) {
        issued = c + 1;   // part A of chunk c is in flight
        if (elect_one()) mbar_arrive_expect_tx(bars + kC2BarLdB + st, 0);   // nothing for B
        __syncwarp();
        break;
      }
      if (elect_one()) load_b(c);
      __syncwarp();
      issued = c + 1;
    }
    if (!ok) {
      // Aborted: the copies of the last two issued chunks land first (each
      // wait bounded on its own; a landed phase reads as complete).
      for (int c = issued > 2 ? issued - 2 : 0; c < issued; ++c) {
        mbar_wait(bars + kC2BarLdA + (c & 1), (c >> 1) & 1);
        mbar_wait(bars + kC2BarLdB + (c & 1), (c >> 1) & 1);
      }
    }
  } else if (warp == kC2M1Warp) {
    // ------------------------------------------------ M1 warp
    bool ok = true;
    // Rows past the sequence end of a short chunk's tile (they hold the next
    // sequence's tokens): zero them before a tensor-core read.
    auto zero_rows = [&](uint8_t* tile, int nblk, int clen) {
      const int nrow = kChunk - clen;
      for (int e = lane; e < nblk * nrow * 8; e += 32) {
        const int blk = e / (nrow * 8);
        const int r = clen + (e >> 3) % nrow;
        *reinterpret_cast<uint4*>(tile + blk * 8192 + sw128_off(r, e & 7)) =
            make_uint4(0, 0, 0, 0);
      }
      fence_proxy_async_smem();
      __syncwarp();
    };
    for (int c = 0; c < nch; ++c) {
      const int st = c & 1;
      uint8_t* stage = smem + st * L::kStage;
      const int clen = chunk_len(c);
      if (!(ok = warp_wait(kC2BarLdA + st, (c >> 1) & 1, kStatusTmaTimeout))) break;
      if (clen < kChunk && !sp.zero_v) zero_rows(stage + L::kStV, L::kVBlocks, clen);
      // M1 into D_UO[st] once the output warps have read its chunk c - 2 (with
      // zero V there is no M1; the commit then only orders the buffer's reuse)
      if (c >= 2 && !(ok = warp_wait(kC2BarOut + st, ((c - 2) >> 1) & 1, kStatusMmaTimeout)))
        break;
      tc_fence_after();
      if (elect_one()) {
        const uint32_t a_st = smem_u32(stage);
        if (!sp.zero_v) {
#pragma unroll
          for (int s = 0; s < 4; ++s)
            umma_bf16(tmem + L::kTmUO + kVS * st, sdesc_sw128(a_st + L::kStPT + s * 32, 16, 1024),
                      sdesc_sw128(a_st + L::kStV + s * 2048, 8192, 1024), idesc_uo,
                      s > 0 ? 1u : 0u);
        }
        umma_commit(bars + kC2BarM1 + st);
      }
      __syncwarp();
      if (!(ok = warp_wait(kC2BarLdB + st, (c >> 1) & 1, kStatusTmaTimeout))) break;
      if (clen < kChunk) zero_rows(stage + L::kStK, 2, clen);
      if (elect_one()) mbar_arrive(bars + kC2BarKReady + st);
      __syncwarp();
    }
    if (!ok) drain_mma(kC2BarEnd2);
  } else if (warp < kC2StateWarps) {
    // ------------------------------------------------ state warps
    // Every state warp runs all nch iterations and reaches both named
    // barriers each time, also after a failed wait (the work is then
    // skipped): a warp that left early would strand the others there.
    const uint32_t a_sb = smem_u32(smem + L::kOffSB);
    const uint32_t a_vnd = smem_u32(smem + L::kOffVND);
    const uint32_t idesc_s = idesc_bf16_f32(128, kVS, 1, 1);
    bool ok = true;
    // Waits on phases that are normally long complete sit in idle slots of
    // the previous step, off the chain: the gammas of chunk c + 1 and (warp 0)
    // M1 of chunk c + 1 while M3 of chunk c runs, K of chunk c while the
    // v_new epilogue runs.
    float gam_last = 0.f, dec = 0.f;
    auto gammas = [&](int c) {   // chunk c's gamma_last and this row's v_new decay
      ok = ok && warp_wait(kC2BarLdA + (c & 1), (c >> 1) & 1, kStatusTmaTimeout);
      if (ok) {
        const float* gam = reinterpret_cast<const float*>(smem + (c & 1) * L::kStage + L::kStGam);
        const int clen = chunk_len(c), cc = row - 64;
        gam_last = gam[clen - 1];
        dec = (quad >= 2 && cc < clen) ? __expf(gam_last - gam[cc]) : 0.f;
      }
    };
    gammas(0);
    if (warp == 0) ok = ok && warp_wait(kC2BarM1, 0, kStatusMmaTimeout);
    for (int c = 0; c < nch; ++c) {
      const int st = c & 1;
      const uint32_t a_st = smem_u32(smem + st * L::kStage);
      if (warp == 0) {   // M2 (M1 of this chunk is complete), then K of this chunk
        if (ok) {
          tc_fence_after();
#pragma unroll
          for (int s = 0; s < 8; ++s)
            umma_bf16_elect(tmem + L::kTmUO + kVS * st,
                            sdesc_sw128(a_st + L::kStQW + (s >> 2) * 16384 + (s & 3) * 32, 16, 1024),
                            sdesc_sw128(a_sb + s * 2048, 16384, 1024), idesc_uo,
                            (s > 0 || !sp.zero_v) ? 1u : 0u);
          umma_commit_elect(bars + kC2BarUO + st);
        }
        ok = ok && warp_wait(kC2BarKReady + st, (c >> 1) & 1, kStatusTmaTimeout);
      }
      if (quad >= 2) {   // v_new rows -> decayed v_new tile
        ok = ok && warp_wait(kC2BarUO + st, (c >> 1) & 1, kStatusMmaTimeout);
        if (ok) {
          tc_fence_after();
          float r[kCols];
          if constexpr (kCols == 32) {
            tmem_ld32(tmem + L::kTmUO + kVS * st + tm_lane + kCols * half, r);
          } else {
            tmem_ld64(tmem + L::kTmUO + kVS * st + tm_lane + kCols * half, r);
          }
          tmem_wait_ld();
          st_cols_bf16(smem + L::kOffVND, 8192, row - 64, r, dec);
          fence_proxy_async_smem();
        }
      }
      tc_fence_before();
      state_sync(1);
      const float decay = __expf(gam_last);
      if (warp == 0 && ok) {   // M3; the record part of the stage is then free
        tc_fence_after();
#pragma unroll
        for (int s = 0; s < 4; ++s)
          umma_bf16_elect(tmem + L::kTmS4, sdesc_sw128(a_st + L::kStK + s * 2048, 8192, 1024),
                          sdesc_sw128(a_vnd + s * 2048, 8192, 1024), idesc_s, s > 0 ? 1u : 0u);
        umma_commit_elect(bars + kC2BarS);
        if (elect_one()) mbar_arrive(bars + kC2BarFreeA + st);
        __syncwarp();
      }
      if (c + 1 < nch) {
        gammas(c + 1);
        if (warp == 0) ok = ok && warp_wait(kC2BarM1 + (st ^ 1), ((c + 1) >> 1) & 1, kStatusMmaTimeout);
      }
      ok = ok && warp_wait(kC2BarS, c & 1, kStatusMmaTimeout);
      if (ok) {   // S_s^T = e^{gamma_last} S_s^T + D_S4
        tc_fence_after();
        float r[kCols];
        if constexpr (kCols == 32) {
          tmem_ld32(tmem + L::kTmS4 + tm_lane + kCols * half, r);
        } else {
          tmem_ld64(tmem + L::kTmS4 + tm_lane + kCols * half, r);
        }
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < kCols; ++j) sreg[j] = fmaf(decay, sreg[j], r[j]);
        st_cols_bf16(smem + L::kOffSB, 16384, row, sreg, 1.0f);
        fence_proxy_async_smem();
        if (warp == 0) {
          if (elect_one()) mbar_arrive(bars + kC2BarFreeB + st);
          __syncwarp();
        }
      }
      tc_fence_before();
      state_sync(2);
    }
    if (warp == 0 && *abort_flag) drain_mma(kC2BarEnd);
  } else {
    // ------------------------------------------------ output warps (TMEM lanes 0-63)
    const int orow = (warp - kC2StateWarps) * 32 + lane;
    for (int c = 0; c < nch; ++c) {
      const int st = c & 1;
      if (!warp_wait(kC2BarUO + st, (c >> 1) & 1, kStatusMmaTimeout)) break;
      tc_fence_after();
      // kVS / 64 blocks of 64 columns; D_UO[st] is released after the last
      // block's TMEM read, before that block's global stores
      const bool write = p.out && orow < chunk_len(c);
      __nv_bfloat16* o = p.out + (static_cast<size_t>(cstart0 + 64 * c + orow) * p.h_v + head) *
                                     kHeadDim + kVS * vs;
#pragma unroll
      for (int b = 0; b < L::kVBlocks; ++b) {
        float r[64];
        tmem_ld64(tmem + L::kTmUO + kVS * st + tm_lane + 64 * b, r);
        if (b == L::kVBlocks - 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(bars + kC2BarOut + st);
        }
        if (write) {
#pragma unroll
          for (int cc = 0; cc < 8; ++cc) {
            uint4 u;
            u.x = pack_bf16x2(p.scale * r[8 * cc + 0], p.scale * r[8 * cc + 1]);
            u.y = pack_bf16x2(p.scale * r[8 * cc + 2], p.scale * r[8 * cc + 3]);
            u.z = pack_bf16x2(p.scale * r[8 * cc + 4], p.scale * r[8 * cc + 5]);
            u.w = pack_bf16x2(p.scale * r[8 * cc + 6], p.scale * r[8 * cc + 7]);
            *reinterpret_cast<uint4*>(o + 64 * b + 8 * cc) = u;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const bool aborted = *abort_flag != 0;
  if (!aborted && warp < kC2StateWarps) {
#pragma unroll
    for (int j = 0; j < kCols; ++j)
      p.new_state[sbase + static_cast<size_t>(kCols * half + j) * kHeadDim + row] = sreg[j];
  }
  return !aborted;
  };

  if constexpr (kScan) {
    const int w = sp.c_lo / sp.window;
    const int s_lo = sp.win_seq[2 * w], s_end = sp.win_seq[2 * w + 1];
    if (sp.group <= 1 && sp.num_seqs > 1 && sp.num_seqs <= kOrderMax) {
      // the window's candidates in the longest-first order of the chunk-table
      // kernel: the rows' first sequences are the window's long ones
      int k = 0;
      for (int r = 0; r < sp.num_seqs; ++r) {
        const int seq = sp.order[r];
        if (seq < s_lo || seq >= s_end) continue;
        if (k++ % static_cast<int>(gridDim.y) != static_cast<int>(blockIdx.y)) continue;
        if (!run_sequence(seq)) break;
      }
    } else {
      for (int seq = s_lo + static_cast<int>(blockIdx.y); seq < s_end;
           seq += static_cast<int>(gridDim.y))
        if (!run_sequence(seq)) break;
    }
  } else {
    run_sequence(row_seq);
  }
  if (have_tmem) {
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) tmem_dealloc(tmem, L::kTmCols);
  }
}

}  // namespace gdn
