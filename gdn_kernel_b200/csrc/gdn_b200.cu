// C-ABI entry points of the B200 GDN hot path (declared in include/gdn_b200.h):
// host-side validation, TMA tensor-map construction and kernel launches.
// One translation unit so that a single device status word serves every kernel.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <limits>
#include <string>

#include "gdn_b200.h"
#include "decode_kernel.cuh"
#include "prefill_split.cuh"
#include "state_affine_kernel.cuh"

namespace gdn {

__device__ unsigned int g_status;

namespace {

thread_local std::string t_last_error;

int fail(int code, const std::string& msg) {
  t_last_error = msg;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(GDN_B200_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

bool aligned(const void* p, size_t n) { return (reinterpret_cast<uintptr_t>(p) % n) == 0; }

constexpr int kMaxDevices = 64;

// Per-device one-time setup: address of the status word, dynamic smem opt-in.
struct DeviceSetup {
  bool done = false;
  unsigned int* status = nullptr;
  int sm_count = 0;
};
DeviceSetup g_setup[kMaxDevices];
std::mutex g_setup_mu;

int device_sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
  std::lock_guard<std::mutex> lock(g_setup_mu);
  return g_setup[dev].sm_count > 0 ? g_setup[dev].sm_count : 148;
}

int device_setup(unsigned int** status_out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(GDN_B200_ERR_CUDA, "device index out of range");
  std::lock_guard<std::mutex> lock(g_setup_mu);
  DeviceSetup& s = g_setup[dev];
  if (!s.done) {
    void* addr = nullptr;
    e = cudaGetSymbolAddress(&addr, g_status);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(status)");
    e = cudaFuncSetAttribute(gdn_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(kPrefillSmem));
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(prefill smem)");
    e = cudaFuncSetAttribute(gdn_prefill_prep_kernel,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kP1Smem));
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(prep smem)");
    for (auto fn : {gdn_prefill_chain_kernel<64, false>, gdn_prefill_chain_kernel<64, true>}) {
      e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(ChainLayout<64>::kSmem));
      if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(chain smem)");
    }
    for (auto fn : {gdn_prefill_chain_kernel<128, false>, gdn_prefill_chain_kernel<128, true>}) {
      e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(ChainLayout<128>::kSmem));
      if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(chain smem, wide)");
    }
    int sms = 0;
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute(SM count)");
    s.sm_count = sms;
    s.status = static_cast<unsigned int*>(addr);
    s.done = true;
  }
  *status_out = s.status;
  return GDN_B200_OK;
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// Tensor map over a packed [tokens, heads, 128] bf16 tensor; box = 64 tokens x
// 1 head x 64 features (128 bytes, the 128B-swizzle span).
int make_token_map(CUtensorMap* m, const void* base, int heads, long long tokens) {
  EncodeTiledFn enc = get_encode_tiled();
  if (!enc) return fail(GDN_B200_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(kHeadDim), static_cast<cuuint64_t>(heads),
                        static_cast<cuuint64_t>(tokens)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(kHeadDim) * 2,
                           static_cast<cuuint64_t>(heads) * kHeadDim * 2};
  cuuint32_t box[3] = {64, 1, static_cast<cuuint32_t>(kChunk)};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(GDN_B200_ERR_CUDA, "cuTensorMapEncodeTiled failed");
  return GDN_B200_OK;
}

int check_heads(int32_t h_qk, int32_t h_v, int32_t d) {
  if (d != kHeadDim) return fail(GDN_B200_ERR_INVALID_ARGUMENT, "head_dim must be 128");
  if (h_qk <= 0 || h_v <= 0)
    return fail(GDN_B200_ERR_INVALID_ARGUMENT, "head counts must be positive");
  if (h_v % h_qk != 0)
    return fail(GDN_B200_ERR_INVALID_ARGUMENT, "num_v_heads must be a multiple of num_qk_heads");
  return GDN_B200_OK;
}

float resolve_scale(double scale) {
  float s = static_cast<float>(scale);
  if (s == 0.0f) s = 1.0f / std::sqrt(static_cast<float>(kHeadDim));
  return s;
}

}  // namespace
}  // namespace gdn

using namespace gdn;

extern "C" int gdn_b200_decode(const void* q, const void* k, const void* v, const float* state,
                               const float* A_log, const void* a, const float* dt_bias,
                               const void* b, double scale, void* output, float* new_state,
                               int64_t batch, int32_t num_qk_heads, int32_t num_v_heads,
                               int32_t head_dim, void* stream) {
  t_last_error.clear();
  if (int rc = check_heads(num_qk_heads, num_v_heads, head_dim)) return rc;
  if (batch < 0) return fail(GDN_B200_ERR_INVALID_ARGUMENT, "batch must be >= 0");
  if (batch * num_v_heads * decode_ctas_per_head<float>() > 0x7fffffffLL)
    return fail(GDN_B200_ERR_INVALID_ARGUMENT, "batch * num_v_heads exceeds the grid limit");
  if (batch == 0) return GDN_B200_OK;
  if (!q || !k || !v || !A_log || !a || !dt_bias || !b || !output || !new_state)
    return fail(GDN_B200_ERR_INVALID_ARGUMENT, "null pointer argument");
  if (!aligned(q, 8) || !aligned(k, 8) || !aligned(new_state, 16) ||
      (state && !aligned(state, 16)))
    return fail(GDN_B200_ERR_INVALID_ARGUMENT,
                "q/k need 8-byte and state/new_state 16-byte alignment");
  unsigned int* status = nullptr;
  if (int rc = device_setup(&status)) return rc;
  DecodeParams p;
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.k = static_cast<const __nv_bfloat16*>(k);
  p.v = static_cast<const __nv_bfloat16*>(v);
  p.pool = state;              // slot = batch entry (no indices); nullptr = zero state
  p.new_pool = new_state;
  p.inter = nullptr;
  p.read_idx = nullptr;
  p.write_idx = nullptr;
  p.idx_is_int64 = 0;
  p.A_log = A_log;
  p.a = static_cast<const __nv_bfloat16*>(a);
  p.dt_bias = dt_bias;
  p.b = static_cast<const __nv_bfloat16*>(b);
  p.scale = resolve_scale(scale);
  p.out = static_cast<__nv_bfloat16*>(output);
  p.status = status;
  p.pool_size = batch;
  p.T = 1;
  p.h_qk = num_qk_heads;
  p.h_v = num_v_heads;
  launch_decode(p, batch, false, static_cast<cudaStream_t>(stream));
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "decode launch");
  return GDN_B200_OK;
}

extern "C" int gdn_b200_decode_pool(const void* q, const void* k, const void* v,
                                    const void* state_pool, void* new_state_pool,
                                    int32_t state_is_bf16, const void* read_indices,
                                    const void* write_indices, int32_t indices_are_int64,
                                    void* intermediate_states, const float* A_log, const void* a,
                                    const float* dt_bias, const void* b, double scale,
                                    void* output, int64_t batch, int64_t seq_len,
                                    int64_t pool_size, int32_t num_qk_heads, int32_t num_v_heads,
                                    int32_t head_dim, void* stream) {
  t_last_error.clear();
  if (int rc = check_heads(num_qk_heads, num_v_heads, head_dim)) return rc;
  if (batch < 0) return fail(GDN_B200_ERR_INVALID_ARGUMENT, "batch must be >= 0");
  if (seq_len < 1 || seq_len > 0x7fffffffLL)
    return fail(GDN_B200_ERR_INVALID_ARGUMENT, "seq_len must be in [1, 2^31)");
  if (batch * num_v_heads * decode_ctas_per_head<float>() > 0x7fffffffLL)
    return fail(GDN_B200_ERR_INVALID_ARGUMENT, "batch * num_v_heads exceeds the grid limit");
  if (batch == 0) return GDN_B200_OK;
  if (pool_size < 1) return fail(GDN_B200_ERR_INVALID_ARGUMENT, "pool_size must be >= 1");
  if (!aligned(v, 2) || !aligned(a, 2) || !aligned(b, 2))
    return fail(GDN_B200_ERR_INVALID_ARGUMENT, "v/a/b need 2-byte alignment");
  if (!q || !k || !v || !state_pool || !new_state_pool || !read_indices || !A_log || !a ||
      !dt_bias || !b || !output)
    return fail(GDN_B200_ERR_INVALID_ARGUMENT, "null pointer argument");
  if (!aligned(q, 16) || !aligned(k, 16) || !aligned(state_pool, 16) ||
      !aligned(new_state_pool, 16) || (intermediate_states && !aligned(intermediate_states, 16)))
    return fail(GDN_B200_ERR_INVALID_ARGUMENT, "q/k and the state buffers need 16-byte alignment");
  unsigned int* status = nullptr;
  if (int rc = device_setup(&status)) return rc;
  DecodeParams p;
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.k = static_cast<const __nv_bfloat16*>(k);
  p.v = static_cast<const __nv_bfloat16*>(v);
  p.pool = state_pool;
  p.new_pool = new_state_pool;
  p.inter = intermediate_states;
  p.read_idx = read_indices;
  p.write_idx = write_indices;
  p.idx_is_int64 = indices_are_int64 ? 1 : 0;
  p.A_log = A_log;
  p.a = static_cast<const __nv_bfloat16*>(a);
  p.dt_bias = dt_bias;
  p.b = static_cast<const __nv_bfloat16*>(b);
  p.scale = resolve_scale(scale);
  p.out = static_cast<__nv_bfloat16*>(output);
  p.status = status;
  p.pool_size = pool_size;
  p.T = static_cast<int>(seq_len);
  p.h_qk = num_qk_heads;
  p.h_v = num_v_heads;
  launch_decode(p, batch, state_is_bf16 != 0, static_cast<cudaStream_t>(stream));
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "pooled decode launch");
  return GDN_B200_OK;
}

extern "C" int gdn_b200_state_affine(const float* state, const float* transfer,
                                     const float* offset, float* out, int64_t num_heads,
                                     void* stream) {
  t_last_error.clear();
  if (num_heads < 0 || num_heads > 65535)
    return fail(GDN_B200_ERR_INVALID_ARGUMENT, "num_heads must be in [0, 65535]");
  if (num_heads == 0) return GDN_B200_OK;
  if (!offset || !out || (state && !transfer))
    return fail(GDN_B200_ERR_INVALID_ARGUMENT, "null pointer argument");
  if (out == state || out == transfer)
    return fail(GDN_B200_ERR_INVALID_ARGUMENT, "out must not alias state or transfer");
  const dim3 grid((kHeadDim / kAffineTile) * (kHeadDim / kAffineTile),
                  static_cast<unsigned>(num_heads));
  gdn_state_affine_kernel<<<grid, kAffineThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      state, transfer, offset, out);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "state affine launch");
  return GDN_B200_OK;
}

namespace gdn {
namespace {

// Shared argument checks and parameter setup of both prefill entry points.
int prefill_setup(const void* q, const void* k, const void* v, const float* state,
                  const float* A_log, const void* a, const float* dt_bias, const void* b,
                  const void* cu_seqlens, int32_t cu_seqlens_is_int64, double scale, void* output,
                  float* new_state, int64_t num_seqs, int64_t total_tokens, int32_t num_qk_heads,
                  int32_t num_v_heads, int32_t head_dim, PrefillParams* p, CUtensorMap* tq,
                  CUtensorMap* tk, CUtensorMap* tv) {
  if (int rc = check_heads(num_qk_heads, num_v_heads, head_dim)) return rc;
  if (num_seqs < 0 || total_tokens < 0)
    return fail(GDN_B200_ERR_INVALID_ARGUMENT, "num_seqs and total_tokens must be >= 0");
  if (num_seqs > 65535)
    return fail(GDN_B200_ERR_INVALID_ARGUMENT, "num_seqs exceeds 65535");
  if (total_tokens > 0x7fffffffLL - kChunk)
    return fail(GDN_B200_ERR_INVALID_ARGUMENT, "total_tokens exceeds the int32 TMA coordinate range");
  if (num_seqs == 0) return GDN_B200_OK;
  if (!cu_seqlens || !A_log || !dt_bias || !new_state)
    return fail(GDN_B200_ERR_INVALID_ARGUMENT, "null pointer argument");
  if (total_tokens > 0 && (!q || !k || !v || !a || !b || !output))
    return fail(GDN_B200_ERR_INVALID_ARGUMENT, "null token tensor with total_tokens > 0");
  if ((total_tokens > 0 && (!aligned(q, 16) || !aligned(k, 16) || !aligned(v, 16) ||
                            !aligned(output, 16))) ||
      !aligned(new_state, 16) || (state && !aligned(state, 16)))
    return fail(GDN_B200_ERR_INVALID_ARGUMENT,
                "q/k/v/output/state/new_state need 16-byte alignment");
  if (!aligned(cu_seqlens, cu_seqlens_is_int64 ? 8 : 4))
    return fail(GDN_B200_ERR_INVALID_ARGUMENT, "cu_seqlens is misaligned");
  unsigned int* status = nullptr;
  if (int rc = device_setup(&status)) return rc;

  // With no tokens every sequence is empty; the maps still need a valid extent,
  // so they describe a one-token view of new_state's (aligned) memory, which no
  // CTA reads because every sequence returns before its first load.
  const long long map_tokens = total_tokens > 0 ? total_tokens : 1;
  const void* qb = total_tokens > 0 ? q : new_state;
  const void* kb = total_tokens > 0 ? k : new_state;
  const void* vb = total_tokens > 0 ? v : new_state;
  if (int rc = make_token_map(tq, qb, total_tokens > 0 ? num_qk_heads : 1, map_tokens)) return rc;
  if (int rc = make_token_map(tk, kb, total_tokens > 0 ? num_qk_heads : 1, map_tokens)) return rc;
  if (int rc = make_token_map(tv, vb, total_tokens > 0 ? num_v_heads : 1, map_tokens)) return rc;

  p->state = state;
  p->A_log = A_log;
  p->a = static_cast<const __nv_bfloat16*>(a);
  p->dt_bias = dt_bias;
  p->b = static_cast<const __nv_bfloat16*>(b);
  p->cu_seqlens = cu_seqlens;
  p->cu_is_int64 = cu_seqlens_is_int64 ? 1 : 0;
  p->total_tokens = total_tokens;
  p->scale = resolve_scale(scale);
  p->out = static_cast<__nv_bfloat16*>(output);
  p->new_state = new_state;
  p->h_qk = num_qk_heads;
  p->h_v = num_v_heads;
  p->status = status;
  return GDN_B200_OK;
}

// Checks shared by the two-stage entry points that take a caller workspace.
int check_two_stage(int64_t num_seqs, int64_t total_tokens, int32_t num_qk_heads,
                    int32_t num_v_heads, int32_t head_dim, const void* workspace,
                    uint64_t workspace_bytes) {
  if (int rc = check_heads(num_qk_heads, num_v_heads, head_dim)) return rc;
  if (num_seqs < 0 || total_tokens < 0)
    return fail(GDN_B200_ERR_INVALID_ARGUMENT, "num_seqs and total_tokens must be >= 0");
  if (num_seqs > 65535) return fail(GDN_B200_ERR_INVALID_ARGUMENT, "num_seqs exceeds 65535");
  if (total_tokens > 0x7fffffffLL - kChunk)
    return fail(GDN_B200_ERR_INVALID_ARGUMENT, "total_tokens exceeds the int32 TMA coordinate range");
  if (num_seqs == 0) return GDN_B200_OK;
  const SplitLayout L = split_layout(num_seqs, total_tokens, num_v_heads);
  if (!workspace || workspace_bytes < L.total || !aligned(workspace, 256))
    return fail(GDN_B200_ERR_INVALID_ARGUMENT,
                "workspace is null, not 256-byte aligned or smaller than "
                "gdn_b200_prefill_workspace_size()");
  if (L.max_chunks > 0x7fffffffLL) return fail(GDN_B200_ERR_INVALID_ARGUMENT, "too many chunks");
  return GDN_B200_OK;
}

SplitParams split_params(const PrefillParams& p, void* workspace, const SplitLayout& L,
                         int64_t num_seqs, int zero_v) {
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  SplitParams sp;
  sp.base = p;
  sp.zero_v = zero_v;
  sp.header = reinterpret_cast<int*>(ws + L.off_header);
  sp.seq_off = reinterpret_cast<int*>(ws + L.off_seq);
  sp.order = reinterpret_cast<int*>(ws + L.off_order);
  sp.table = reinterpret_cast<ChunkInfo*>(ws + L.off_table);
  sp.records = ws + L.off_rec;
  sp.num_seqs = static_cast<int>(num_seqs);
  sp.max_chunks = static_cast<int>(L.max_chunks);
  sp.ring_rows = static_cast<int>(L.max_chunks);
  sp.group = 1;
  sp.block = 1;
  sp.window = 0;
  sp.scan = 0;
  sp.wait_limit_ns = 0;
  sp.withhold_from = -1;
  sp.win_seq = reinterpret_cast<int*>(ws + L.off_win);
  sp.c_lo = 0;
  sp.c_hi = std::numeric_limits<int>::max();
  sp.wait_table = 0;
  return sp;
}

// The prep kernel over `items` (chunk, v-head) items of sp's chunk window,
// persistent on at most `max_ctas` CTAs.  With `overlap` it is launched to
// start while the chain kernel before it in the stream still runs (that
// kernel's CTAs trigger it once all are resident; it completes after it).
void launch_prep(const SplitParams& sp, const CUtensorMap& tq, const CUtensorMap& tk,
                 long long items, long long max_ctas, bool overlap, cudaStream_t st) {
  const long long ctas = std::min(items, max_ctas);
  if (ctas <= 0) return;
  if (!overlap) {
    gdn_prefill_prep_kernel<<<static_cast<unsigned>(ctas), kPrefillThreads, kP1Smem, st>>>(tq, tk,
                                                                                          sp);
    return;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(ctas));
  cfg.blockDim = dim3(kPrefillThreads);
  cfg.dynamicSmemBytes = kP1Smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, gdn_prefill_prep_kernel, tq, tk, sp) != cudaSuccess) {
    // Without the overlap the grid simply runs after the chain before it (same
    // results); a launch that fails again leaves its error for the caller.
    (void)cudaGetLastError();
    gdn_prefill_prep_kernel<<<static_cast<unsigned>(ctas), kPrefillThreads, kP1Smem, st>>>(tq, tk,
                                                                                          sp);
  }
}

// The prep grid that follows the chunk-table kernel is launched with
// programmatic serialization and waits for the table inside (wait_table), so
// its launch and setup overlap the table kernel.
void launch_table_then_prep(const SplitParams& sp, const CUtensorMap& tq, const CUtensorMap& tk,
                            long long items, long long max_ctas, cudaStream_t st) {
  gdn_chunk_table_kernel<<<1, kTableThreads, 0, st>>>(sp);
  SplitParams first = sp;
  first.wait_table = 1;
  launch_prep(first, tq, tk, items, max_ctas, true, st);
}

// Chunk table and per-(chunk, v-head) records into the workspace.
void launch_prepare(const SplitParams& sp, const CUtensorMap& tq, const CUtensorMap& tk,
                    const SplitLayout& L, int32_t num_v_heads, cudaStream_t st) {
  // Persistent: two CTAs per SM (at most one per item) walk the items.
  launch_table_then_prep(sp, tq, tk, L.max_chunks * static_cast<long long>(num_v_heads),
                         2LL * device_sm_count(), st);
}

// The state recurrence over a prepared workspace (reads it only).  A chain
// CTA owns all 128 of a head's V columns or 64 (two CTAs per head).  The wide
// CTA does both halves' work in about 1.2x the time per chunk (measured on
// B200) and loads each record once instead of twice; the narrow one spreads
// few (sequence, head) pairs n over more SMs.  With one chain CTA per SM, the
// narrow form takes ceil(2n / SMs) waves of time t and the wide one
// ceil(n / SMs) waves of 1.2 t, so the wide form wins once 2n > SMs.  (The
// one-sequence pieces path keeps the narrow form: its idle SMs run the prep.)
void launch_recur(const SplitParams& sp, const CUtensorMap& tk, const CUtensorMap& tv,
                  int64_t num_seqs, int32_t num_v_heads, cudaStream_t st, bool allow_wide = true,
                  bool pdl = false) {
  // (num_seqs: CTA rows of the grid; with sp.scan each row runs a window's candidates)
  // pdl: launched with programmatic serialization after the prep whose records
  // it reads (which triggers at its start), so the grid's CTAs take SMs as the
  // prep's CTAs, or those of the chain before, retire, and wait inside for the
  // prep's completion; otherwise a plain launch.
  const bool wide = allow_wide && 2 * num_seqs * num_v_heads > static_cast<int64_t>(device_sm_count());
  const dim3 g(static_cast<unsigned>((wide ? 1 : 2) * num_v_heads), static_cast<unsigned>(num_seqs));
  auto go = [&](void (*kern)(const CUtensorMap, const CUtensorMap, const SplitParams),
                uint32_t smem) {
    if (pdl) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = g;
      cfg.blockDim = dim3(kC2Threads);
      cfg.dynamicSmemBytes = smem;
      cfg.stream = st;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      attr[0].val.programmaticStreamSerializationAllowed = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      if (cudaLaunchKernelEx(&cfg, kern, tk, tv, sp) == cudaSuccess) return;
      (void)cudaGetLastError();   // as a plain launch below: the same results
    }
    kern<<<g, kC2Threads, smem, st>>>(tk, tv, sp);
  };
  if (wide)
    go(sp.scan ? gdn_prefill_chain_kernel<128, true> : gdn_prefill_chain_kernel<128, false>,
       ChainLayout<128>::kSmem);
  else
    go(sp.scan ? gdn_prefill_chain_kernel<64, true> : gdn_prefill_chain_kernel<64, false>,
       ChainLayout<64>::kSmem);
}

// A whole two-stage call.  One short-grid sequence (its chain kernel fills at
// most half the SMs) runs in pieces of its chunks instead, so that each
// piece's prep overlaps the previous piece's chain on the SMs the chain
// leaves idle:
//   table | prep(1) on all SMs | chain(1) || prep(2) | chain(2) || prep(3) | ...
// The chain kernel's CTAs take their SMs first (they trigger the overlapping
// prep grid once all are resident, and a prep CTA does not fit beside one),
// and that prep grid is sized to the free SMs.  It completes only after the
// chain it overlaps, so the next chain, launched after it, starts from the
// previous piece's final state (new_state).  Every chunk is computed exactly
// as in one piece.
//
// Piece sizes fall geometrically, n_{i+1} = r n_i, so that the prep of piece
// i+1 on the free SMs takes about as long as the chain of piece i: r is near
// the chain's time per chunk over the overlapped prep's (on B200 at H_v = 32,
// 1.42 us against 1.66 us serialised; 0.90 measured best of 0.80-0.99, all
// within 3 %).  Everything after the first prep then runs at the chain's pace;
// more pieces shrink that first prep but add launch overhead, so the count
// grows with the sequence (one per 32 chunks, 2 to 8).
constexpr long long kPieceMinChunks = 16;   // shorter sequences run in one piece
constexpr double kPieceRatio = 0.90;
constexpr int kPieceMaxCount = 8;
constexpr long long kPieceChunksPer = 32;

void launch_two_stage(const SplitParams& sp, const CUtensorMap& tq, const CUtensorMap& tk,
                      const CUtensorMap& tv, const SplitLayout& L, int64_t num_seqs,
                      int64_t total_tokens, int32_t num_v_heads, cudaStream_t st) {
  const int sms = device_sm_count();
  const long long chain_ctas = 2LL * num_v_heads * num_seqs;
  const long long nch = (total_tokens + kChunk - 1) / kChunk;   // the sequence's at most
  if (num_seqs != 1 || 2 * chain_ctas > sms || nch < kPieceMinChunks) {
    launch_prepare(sp, tq, tk, L, num_v_heads, st);
    launch_recur(sp, tk, tv, num_seqs, num_v_heads, st);
    return;
  }
  const int count = static_cast<int>(
      std::max<long long>(2, std::min<long long>(kPieceMaxCount, nch / kPieceChunksPer)));
  // piece i ends after a share (1 - r^{i+1}) / (1 - r^count) of the chunks
  const double rk = std::pow(kPieceRatio, count);
  int lo = 0;
  for (int i = 0; i < count; ++i) {
    const double end = (1.0 - std::pow(kPieceRatio, i + 1)) / (1.0 - rk);
    const int hi = i + 1 == count ? std::numeric_limits<int>::max()
                                  : std::max(lo + 1, static_cast<int>(std::lround(nch * end)));
    SplitParams piece = sp;
    piece.c_lo = lo;   // a later piece continues from new_state (the chain kernel's rule)
    piece.c_hi = hi;
    const long long items = (std::min<long long>(hi, nch) - lo) * num_v_heads;
    if (i == 0)
      launch_table_then_prep(piece, tq, tk, items, 2LL * sms, st);
    else
      launch_prep(piece, tq, tk, items, 2LL * (sms - chain_ctas), true, st);
    // The first piece's chain is a plain launch: launched by programmatic
    // serialization after the first prep, one sequence ran slower on B200
    // (8,192 tokens 255 -> 270 us, 65,536 tokens 1.67 -> 1.85 ms).
    launch_recur(piece, tk, tv, num_seqs, num_v_heads, st, true, i > 0);
    lo = hi;
  }
}

// A two-stage call whose records do not all fit the record rows of the
// workspace (a ring of sp.ring_rows rows): consecutive windows of W table
// chunks, the records of chunk g in row g % ring_rows.  With one sequence W =
// ring_rows / 2, so that a window's records fill one half of the ring while
// the chain of the window before it reads the other half; with several, W =
// ring_rows (below).  The host knows only an upper bound
// of the chunk count (ceil(T / 64) + N); windows past the table's real end
// find no items and no chunks.
//  * One sequence: as in the one-sequence pieces, the prep of window i + 1 is
//    launched to overlap the chain of window i on the SMs that chain (64-column
//    CTAs) leaves free, and completes only after it; the prep of window i + 2
//    starts after the chain of window i + 1 has started, i.e. after the chain
//    of window i (the last reader of its half) has completed.
//  * Several sequences: the table interleaves groups of K sequences (K H_v
//    chain CTAs fill the SMs once) in rounds of W / K chunks per member, so
//    each window holds about W / K consecutive chunks of each of K sequences
//    and its chain runs them all at once; the chain then fills the GPU, so
//    each window's prep runs on all SMs after the previous chain.  A window's
//    records (W H_v records) are read back while still in L2.
void launch_windows(const SplitParams& sp0, const CUtensorMap& tq, const CUtensorMap& tk,
                    const CUtensorMap& tv, const SplitLayout& L, int64_t num_seqs,
                    int32_t num_v_heads, cudaStream_t st) {
  const int sms = device_sm_count();
  SplitParams sp = sp0;
  const bool interleave = num_seqs > 1;
  // One sequence: half the ring per window, so that a window's prep fills one
  // half while the chain of the window before reads the other.  Several
  // sequences: a window's prep follows the previous window's chain (a plain
  // launch), so each window takes the whole ring.
  const long long window = interleave ? sp.ring_rows : sp.ring_rows / 2;
  if (interleave) {
    // Groups of K sequences (K H_v chain CTAs fill the SMs once) are interleaved
    // only when a window cannot hold K sequences of the mean length; otherwise
    // the table stays sequence-major (K = 1): each window then holds whole
    // sequences, which the chain runs side by side (varlen16 through the ring
    // 1.67 -> 1.58 ms on B200), and only a sequence at a window's edge is split.
    const int kfill = std::max(1, std::min<int>(kMaxGroup, sms / std::max(1, num_v_heads)));
    const long long mean = std::max<long long>(1, (L.max_chunks - num_seqs) / num_seqs);
    sp.group = mean * kfill > window ? kfill : 1;
    sp.block = static_cast<int>(std::max<long long>(1, window / sp.group));
    sp.window = static_cast<int>(window);
  }
  const long long free_ctas = 2LL * std::max(1, sms - 2 * num_v_heads);
  for (long long lo = 0, i = 0; lo < L.max_chunks; lo += window, ++i) {
    SplitParams win = sp;
    win.c_lo = static_cast<int>(lo);
    win.c_hi = static_cast<int>(std::min<long long>(lo + window, L.max_chunks));
    const long long items = (win.c_hi - win.c_lo) * static_cast<long long>(num_v_heads);
    if (i == 0)
      launch_table_then_prep(win, tq, tk, items, 2LL * sms, st);
    else if (interleave)
      launch_prep(win, tq, tk, items, 2LL * sms, false, st);
    else
      launch_prep(win, tq, tk, items, free_ctas, true, st);
    if (!interleave) {
      launch_recur(win, tk, tv, num_seqs, num_v_heads, st, false, i > 0);
    } else if (i == 0) {
      // every sequence gets a CTA row once (empty sequences copy their state)
      launch_recur(win, tk, tv, num_seqs, num_v_heads, st, true, true);
    } else {
      // CTA rows walk the window's candidate sequences: about as many rows as
      // a window holds sequences of the mean length, plus a partial group at
      // either end (more candidates loop over the rows).
      win.scan = 1;
      const long long mean = std::max<long long>(1, (L.max_chunks - num_seqs) / num_seqs);
      const long long rows =
          std::min<long long>(num_seqs, std::max<long long>(sp.group, window / mean + 2 * sp.group));
      launch_recur(win, tk, tv, rows, num_v_heads, st, true, true);
    }
  }
}

// ---------------------------------------------------------------- record ring
// The reference's prefill `kernel` takes no workspace and allocates nothing
// (ref solution/cuda/kernel_prefill.cu:300-337).  gdn_b200_prefill keeps that
// contract at the speed of the two-stage path: its workspace is a record ring
// that is part of this library's device image (GDN_B200_PREFILL_RING_BYTES on
// every GPU that loads the library, held until the process exits).  The chunk
// tables take its front; the rest holds rows of H_v records.  A problem whose
// records all fit runs exactly as with a caller workspace; a larger one runs
// in windows (launch_windows).  Calls on different streams hand the ring over
// through an event: each call's stream waits for the previous call's last
// kernel, and the host never blocks.  (A stream under graph capture skips
// that handoff; captured calls must not overlap other calls on the device.)
static __device__ __align__(1024) uint8_t g_prefill_ring[GDN_B200_PREFILL_RING_BYTES];

struct RingState {
  void* ptr = nullptr;          // device address of g_prefill_ring on this device
  cudaEvent_t done = nullptr;   // recorded after the last call's final kernel
  bool recorded = false;
};
RingState g_ring[kMaxDevices];
std::mutex g_ring_mu;

}  // namespace
}  // namespace gdn

extern "C" int gdn_b200_prefill(const void* q, const void* k, const void* v, const float* state,
                                const float* A_log, const void* a, const float* dt_bias,
                                const void* b, const void* cu_seqlens,
                                int32_t cu_seqlens_is_int64, double scale, void* output,
                                float* new_state, int64_t num_seqs, int64_t total_tokens,
                                int32_t num_qk_heads, int32_t num_v_heads, int32_t head_dim,
                                void* stream) {
  t_last_error.clear();
  PrefillParams p;
  CUtensorMap tq, tk, tv;
  if (int rc = prefill_setup(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, cu_seqlens_is_int64,
                             scale, output, new_state, num_seqs, total_tokens, num_qk_heads,
                             num_v_heads, head_dim, &p, &tq, &tk, &tv))
    return rc;
  if (num_seqs == 0) return GDN_B200_OK;
  // Ring geometry: the tables first, then as many record rows as fit.
  const SplitLayout front = split_layout(num_seqs, total_tokens, num_v_heads, 0, true);
  const uint64_t row_bytes = static_cast<uint64_t>(num_v_heads) * kRecBytes;
  const uint64_t ring = GDN_B200_PREFILL_RING_BYTES;
  const long long rows =
      front.off_rec < ring ? static_cast<long long>((ring - front.off_rec) / row_bytes) : 0;
  if (rows < 2)
    return fail(GDN_B200_ERR_INVALID_ARGUMENT,
                "problem too large for the prefill record ring (its chunk tables or two rows "
                "of records do not fit); use gdn_b200_prefill_ws with a caller workspace");
  if (front.max_chunks > 0x7fffffffLL) return fail(GDN_B200_ERR_INVALID_ARGUMENT, "too many chunks");
  const long long use_rows = std::min<long long>(rows, front.max_chunks);
  const SplitLayout L = split_layout(num_seqs, total_tokens, num_v_heads, use_rows, true);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  std::lock_guard<std::mutex> lock(g_ring_mu);   // one ring user enqueues at a time
  RingState& R = g_ring[dev];
  if (!R.ptr) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_prefill_ring);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(prefill record ring)");
    e = cudaEventCreateWithFlags(&R.done, cudaEventDisableTiming);
    if (e != cudaSuccess) return cuda_fail(e, "cudaEventCreate(record ring)");
    R.ptr = ptr;
  }
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  e = cudaStreamIsCapturing(st, &cap);
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamIsCapturing");
  const bool handoff = cap == cudaStreamCaptureStatusNone;
  if (handoff && R.recorded && (e = cudaStreamWaitEvent(st, R.done, 0)) != cudaSuccess)
    return cuda_fail(e, "cudaStreamWaitEvent(record ring)");
  SplitParams sp = split_params(p, R.ptr, L, num_seqs, 0);
  sp.ring_rows = static_cast<int>(use_rows);
  if (use_rows >= L.max_chunks)
    launch_two_stage(sp, tq, tk, tv, L, num_seqs, total_tokens, num_v_heads, st);
  else
    launch_windows(sp, tq, tk, tv, L, num_seqs, num_v_heads, st);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "prefill (record ring) launch");
  if (handoff) {
    if ((e = cudaEventRecord(R.done, st)) != cudaSuccess)
      return cuda_fail(e, "cudaEventRecord(record ring)");
    R.recorded = true;
  }
  return GDN_B200_OK;
}

extern "C" int gdn_b200_prefill_fused(const void* q, const void* k, const void* v,
                                      const float* state,
                                const float* A_log, const void* a, const float* dt_bias,
                                const void* b, const void* cu_seqlens,
                                int32_t cu_seqlens_is_int64, double scale, void* output,
                                float* new_state, int64_t num_seqs, int64_t total_tokens,
                                int32_t num_qk_heads, int32_t num_v_heads, int32_t head_dim,
                                void* stream) {
  t_last_error.clear();
  PrefillParams p;
  CUtensorMap tq, tk, tv;
  if (int rc = prefill_setup(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, cu_seqlens_is_int64,
                             scale, output, new_state, num_seqs, total_tokens, num_qk_heads,
                             num_v_heads, head_dim, &p, &tq, &tk, &tv))
    return rc;
  if (num_seqs == 0) return GDN_B200_OK;
  const dim3 grid(static_cast<unsigned>(num_v_heads), static_cast<unsigned>(num_seqs));
  gdn_prefill_kernel<<<grid, kPrefillThreads, kPrefillSmem, static_cast<cudaStream_t>(stream)>>>(
      tq, tk, tv, p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "prefill launch");
  return GDN_B200_OK;
}

extern "C" uint64_t gdn_b200_prefill_workspace_size(int64_t num_seqs, int64_t total_tokens,
                                                    int32_t num_v_heads) {
  if (num_seqs <= 0 || total_tokens < 0 || num_v_heads <= 0) return 0;
  return split_layout(num_seqs, total_tokens, num_v_heads).total;
}

extern "C" int gdn_b200_prefill_ws(const void* q, const void* k, const void* v,
                                   const float* state, const float* A_log, const void* a,
                                   const float* dt_bias, const void* b, const void* cu_seqlens,
                                   int32_t cu_seqlens_is_int64, double scale, void* output,
                                   float* new_state, int64_t num_seqs, int64_t total_tokens,
                                   int32_t num_qk_heads, int32_t num_v_heads, int32_t head_dim,
                                   void* workspace, uint64_t workspace_bytes, void* stream) {
  t_last_error.clear();
  PrefillParams p;
  CUtensorMap tq, tk, tv;
  if (int rc = prefill_setup(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, cu_seqlens_is_int64,
                             scale, output, new_state, num_seqs, total_tokens, num_qk_heads,
                             num_v_heads, head_dim, &p, &tq, &tk, &tv))
    return rc;
  if (num_seqs == 0) return GDN_B200_OK;
  const SplitLayout L = split_layout(num_seqs, total_tokens, num_v_heads);
  if (!workspace || workspace_bytes < L.total || !aligned(workspace, 256))
    return fail(GDN_B200_ERR_INVALID_ARGUMENT,
                "workspace is null, not 256-byte aligned or smaller than "
                "gdn_b200_prefill_workspace_size()");
  if (L.max_chunks > 0x7fffffffLL)
    return fail(GDN_B200_ERR_INVALID_ARGUMENT, "too many chunks");
  const SplitParams sp = split_params(p, workspace, L, num_seqs, 0);
  launch_two_stage(sp, tq, tk, tv, L, num_seqs, total_tokens, num_v_heads,
                   static_cast<cudaStream_t>(stream));
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "prefill (two-stage) launch");
  return GDN_B200_OK;
}

extern "C" int gdn_b200_prefill_prepare(const void* q, const void* k, const float* A_log,
                                        const void* a, const float* dt_bias, const void* b,
                                        const void* cu_seqlens, int32_t cu_seqlens_is_int64,
                                        int64_t num_seqs, int64_t total_tokens,
                                        int32_t num_qk_heads, int32_t num_v_heads,
                                        int32_t head_dim, void* workspace,
                                        uint64_t workspace_bytes, void* stream) {
  t_last_error.clear();
  if (int rc = check_two_stage(num_seqs, total_tokens, num_qk_heads, num_v_heads, head_dim,
                               workspace, workspace_bytes))
    return rc;
  if (num_seqs == 0) return GDN_B200_OK;
  if (!cu_seqlens || !A_log || !dt_bias)
    return fail(GDN_B200_ERR_INVALID_ARGUMENT, "null pointer argument");
  if (total_tokens > 0 && (!q || !k || !a || !b))
    return fail(GDN_B200_ERR_INVALID_ARGUMENT, "null token tensor with total_tokens > 0");
  if (total_tokens > 0 && (!aligned(q, 16) || !aligned(k, 16)))
    return fail(GDN_B200_ERR_INVALID_ARGUMENT, "q/k need 16-byte alignment");
  if (!aligned(cu_seqlens, cu_seqlens_is_int64 ? 8 : 4))
    return fail(GDN_B200_ERR_INVALID_ARGUMENT, "cu_seqlens is misaligned");
  unsigned int* status = nullptr;
  if (int rc = device_setup(&status)) return rc;
  CUtensorMap tq, tk;
  const long long map_tokens = total_tokens > 0 ? total_tokens : 1;
  const void* qb = total_tokens > 0 ? q : workspace;
  const void* kb = total_tokens > 0 ? k : workspace;
  const int hm = total_tokens > 0 ? num_qk_heads : 1;
  if (int rc = make_token_map(&tq, qb, hm, map_tokens)) return rc;
  if (int rc = make_token_map(&tk, kb, hm, map_tokens)) return rc;
  PrefillParams p{};
  p.A_log = A_log;
  p.a = static_cast<const __nv_bfloat16*>(a);
  p.dt_bias = dt_bias;
  p.b = static_cast<const __nv_bfloat16*>(b);
  p.cu_seqlens = cu_seqlens;
  p.cu_is_int64 = cu_seqlens_is_int64 ? 1 : 0;
  p.total_tokens = total_tokens;
  p.h_qk = num_qk_heads;
  p.h_v = num_v_heads;
  p.status = status;
  const SplitLayout L = split_layout(num_seqs, total_tokens, num_v_heads);
  const SplitParams sp = split_params(p, workspace, L, num_seqs, 0);
  launch_prepare(sp, tq, tk, L, num_v_heads, static_cast<cudaStream_t>(stream));
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "prefill prepare launch");
  return GDN_B200_OK;
}

namespace gdn {
namespace {
int recur_impl(const void* k, const void* v, const float* state, double scale, void* output,
               float* new_state, int64_t num_seqs, int64_t total_tokens, int32_t num_qk_heads,
               int32_t num_v_heads, int32_t head_dim, const void* workspace,
               uint64_t workspace_bytes, void* stream, unsigned long long wait_limit_ns,
               int withhold_from) {
  if (int rc = check_two_stage(num_seqs, total_tokens, num_qk_heads, num_v_heads, head_dim,
                               workspace, workspace_bytes))
    return rc;
  if (num_seqs == 0) return GDN_B200_OK;
  if (!new_state) return fail(GDN_B200_ERR_INVALID_ARGUMENT, "null pointer argument");
  if (total_tokens > 0 && !k)
    return fail(GDN_B200_ERR_INVALID_ARGUMENT, "null k with total_tokens > 0");
  if ((total_tokens > 0 && (!aligned(k, 16) || (v && !aligned(v, 16)) ||
                            (output && !aligned(output, 16)))) ||
      !aligned(new_state, 16) || (state && !aligned(state, 16)))
    return fail(GDN_B200_ERR_INVALID_ARGUMENT,
                "k/v/output/state/new_state need 16-byte alignment");
  unsigned int* status = nullptr;
  if (int rc = device_setup(&status)) return rc;
  CUtensorMap tk, tv;
  const long long map_tokens = total_tokens > 0 ? total_tokens : 1;
  const void* kb = total_tokens > 0 ? k : workspace;
  if (int rc = make_token_map(&tk, kb, total_tokens > 0 ? num_qk_heads : 1, map_tokens)) return rc;
  // With zero V the V map is never read; it describes k's memory to stay valid.
  if (total_tokens > 0 && v) {
    if (int rc = make_token_map(&tv, v, num_v_heads, map_tokens)) return rc;
  } else {
    tv = tk;
  }
  PrefillParams p{};
  p.state = state;
  p.total_tokens = total_tokens;
  p.scale = resolve_scale(scale);
  p.out = static_cast<__nv_bfloat16*>(output);
  p.new_state = new_state;
  p.h_qk = num_qk_heads;
  p.h_v = num_v_heads;
  p.status = status;
  const SplitLayout L = split_layout(num_seqs, total_tokens, num_v_heads);
  SplitParams sp =
      split_params(p, const_cast<void*>(workspace), L, num_seqs, v == nullptr ? 1 : 0);
  sp.wait_limit_ns = wait_limit_ns;
  sp.withhold_from = withhold_from;
  launch_recur(sp, tk, tv, num_seqs, num_v_heads, static_cast<cudaStream_t>(stream));
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "prefill recurrence launch");
  return GDN_B200_OK;
}
}  // namespace
}  // namespace gdn

extern "C" int gdn_b200_prefill_recur(const void* k, const void* v, const float* state,
                                      double scale, void* output, float* new_state,
                                      int64_t num_seqs, int64_t total_tokens,
                                      int32_t num_qk_heads, int32_t num_v_heads,
                                      int32_t head_dim, const void* workspace,
                                      uint64_t workspace_bytes, void* stream) {
  t_last_error.clear();
  return recur_impl(k, v, state, scale, output, new_state, num_seqs, total_tokens, num_qk_heads,
                    num_v_heads, head_dim, workspace, workspace_bytes, stream, 0, -1);
}

extern "C" int gdn_b200_selftest_prefill_abort(uint64_t limit_ns, const void* k, const void* v,
                                               const float* state, void* output,
                                               float* new_state, int64_t num_seqs,
                                               int64_t total_tokens, int32_t num_qk_heads,
                                               int32_t num_v_heads, int32_t head_dim,
                                               const void* workspace, uint64_t workspace_bytes,
                                               void* stream) {
  t_last_error.clear();
  if (limit_ns == 0 || limit_ns > 1000000000ull)
    return fail(GDN_B200_ERR_INVALID_ARGUMENT, "limit_ns must be in (0, 1e9]");
  return recur_impl(k, v, state, 0.0, output, new_state, num_seqs, total_tokens, num_qk_heads,
                    num_v_heads, head_dim, workspace, workspace_bytes, stream, limit_ns, 2);
}

// ---------------------------------------------------------------- allocation-free prefill
// Some callers of this library cannot allocate device memory: a host bound to
// the reference's fixed `kernel` argument list has no slot to pass a workspace
// in, a plugin host may own all device memory through its own allocator and
// forbid raw cudaMalloc, and a latency-critical serving loop may not accept
// the cost and implicit synchronisation of an allocation on its hot path.
// gdn_b200_prefill_static serves them from a scratch array that is part of
// this library's device image: every GPU that loads the library reserves
// GDN_B200_PREFILL_STATIC_SCRATCH_BYTES for it until the process exits.
namespace gdn {
namespace {

static __device__ __align__(256) uint8_t g_prefill_static_scratch[GDN_B200_PREFILL_STATIC_SCRATCH_BYTES];

// Device address of the scratch array, looked up once per device with that
// device current.  On the host the array's name only stands in for the symbol;
// it is not a device pointer and must never be passed to a kernel.
void* g_static_scratch_ptr[kMaxDevices];
std::mutex g_static_scratch_mu;

int static_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(GDN_B200_ERR_CUDA, "device index out of range");
  std::lock_guard<std::mutex> lock(g_static_scratch_mu);
  if (!g_static_scratch_ptr[dev]) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_prefill_static_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(prefill static scratch)");
    g_static_scratch_ptr[dev] = ptr;
  }
  *out = g_static_scratch_ptr[dev];
  return GDN_B200_OK;
}

}  // namespace
}  // namespace gdn

extern "C" int gdn_b200_prefill_static(const void* q, const void* k, const void* v,
                                       const float* state, const float* A_log, const void* a,
                                       const float* dt_bias, const void* b,
                                       const void* cu_seqlens, int32_t cu_seqlens_is_int64,
                                       double scale, void* output, float* new_state,
                                       int64_t num_seqs, int64_t total_tokens,
                                       int32_t num_qk_heads, int32_t num_v_heads,
                                       int32_t head_dim, void* stream) {
  t_last_error.clear();
  // The extent checks of the workspace path come first, so that a bad size is
  // reported as such and not as "too large for the scratch".
  if (int rc = check_heads(num_qk_heads, num_v_heads, head_dim)) return rc;
  if (num_seqs < 0 || total_tokens < 0)
    return fail(GDN_B200_ERR_INVALID_ARGUMENT, "num_seqs and total_tokens must be >= 0");
  if (num_seqs > 65535) return fail(GDN_B200_ERR_INVALID_ARGUMENT, "num_seqs exceeds 65535");
  if (total_tokens > 0x7fffffffLL - kChunk)
    return fail(GDN_B200_ERR_INVALID_ARGUMENT, "total_tokens exceeds the int32 TMA coordinate range");
  if (num_seqs == 0) return GDN_B200_OK;
  const uint64_t need = gdn_b200_prefill_workspace_size(num_seqs, total_tokens, num_v_heads);
  if (need > GDN_B200_PREFILL_STATIC_SCRATCH_BYTES)
    return fail(GDN_B200_ERR_INVALID_ARGUMENT,
                "problem too large for the static prefill scratch: needs " +
                    std::to_string(need) + " bytes, the limit is " +
                    std::to_string(static_cast<uint64_t>(GDN_B200_PREFILL_STATIC_SCRATCH_BYTES)) +
                    " (use gdn_b200_prefill_ws with a caller workspace)");
  void* scratch = nullptr;
  if (int rc = static_scratch(&scratch)) return rc;
  // Nothing in the scratch has to start at zero: the chunk-table kernel writes
  // every table slot the later kernels read, and the prep kernel writes every
  // record the chain kernel reads, on each call.
  return gdn_b200_prefill_ws(q, k, v, state, A_log, a, dt_bias, b, cu_seqlens, cu_seqlens_is_int64,
                             scale, output, new_state, num_seqs, total_tokens, num_qk_heads,
                             num_v_heads, head_dim, scratch, GDN_B200_PREFILL_STATIC_SCRATCH_BYTES,
                             stream);
}

extern "C" int gdn_b200_device_status(int32_t device, uint32_t* status, int32_t clear) {
  t_last_error.clear();
  if (!status) return fail(GDN_B200_ERR_INVALID_ARGUMENT, "status is null");
  int prev = 0;
  cudaError_t e = cudaGetDevice(&prev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (device != prev && (e = cudaSetDevice(device)) != cudaSuccess)
    return cuda_fail(e, "cudaSetDevice");
  unsigned int v = 0;
  e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemcpyFromSymbol(&v, g_status, sizeof(v));
  if (e == cudaSuccess && clear) {
    const unsigned int zero = 0;
    e = cudaMemcpyToSymbol(g_status, &zero, sizeof(zero));
  }
  if (device != prev) cudaSetDevice(prev);
  if (e != cudaSuccess) return cuda_fail(e, "device status");
  *status = v;
  return GDN_B200_OK;
}

extern "C" const char* gdn_b200_last_error(void) { return t_last_error.c_str(); }

// ---------------------------------------------------------------- bounded-wait self-test
namespace gdn {
// One warp waits on an mbarrier that nothing arrives on, with the same bounded
// wait the prefill kernels use but a caller-chosen limit.  When the limit runs
// out it records kStatusSelftestWait and returns, leaving the context usable.
__global__ void gdn_selftest_wait_kernel(unsigned long long limit_ns, unsigned int* status) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbarrier_init();
  }
  __syncwarp();
  const bool ok = mbar_wait(&bar, 0, limit_ns);
  if (!ok && threadIdx.x == 0) atomicOr(status, kStatusSelftestWait);
}
}  // namespace gdn

extern "C" int gdn_b200_selftest_wait_timeout(uint64_t limit_ns, void* stream) {
  t_last_error.clear();
  if (limit_ns == 0 || limit_ns > 1000000000ull)
    return fail(GDN_B200_ERR_INVALID_ARGUMENT, "limit_ns must be in (0, 1e9]");
  unsigned int* status = nullptr;
  if (int rc = device_setup(&status)) return rc;
  gdn_selftest_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(limit_ns, status);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "self-test launch");
  return GDN_B200_OK;
}

extern "C" int32_t gdn_b200_abi_version(void) { return 103; }

extern "C" int32_t gdn_b200_current_device(void) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    (void)cudaGetLastError();
    return -1;
  }
  return dev;
}
