// dd_api.cu -- host side of libdomino_draft.so: the handle, TMA descriptors,
// the launch sequence of one draft step, and the C ABI of
// include/domino_draft.h.
//
// Launch sequence of one rollout (code/kernel/domino.py:374-431), all on the
// caller's stream, each launch with programmatic dependent launch so that a
// phase's weight stream starts before the previous phase has finished:
//
//   memset(argmax words)
//   Z     gemv  z = parallel_hiddens @ W_z^T (+ fc1 bias)          [B*S, E]
//   P0    cell  h0 = GRU(table[prefix_ids[:, 0]], h = 0)
//   (Pj   gemv  gh = h W_hh^T ; cell h = GRU(table[prefix_ids[:, j]], h))  j = 1..p
//   for t in 0..S-1:
//     SGH gemv  s = h W_s^T -> mid = SiLU(z_t + s) as (hi, lo) rows ;  gh = h W_hh^T
//     FC2 gemv  logit = fc2 (hi + lo) + fc2_bias + base_t -> atomicMax argmax word
//     CELL      token_t -> out ; h = GRU(table[token_t], gh, h)
//
// dd_draft_block replaces the Z launch by one that also computes the base
// logits (lm_head) and the pure-draft prefix argmax.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <type_traits>

#include "../../include/domino_draft.h"
#include "dd_cell.cuh"
#include "dd_gemv.cuh"
#include "dd_gemv_f32.cuh"
#include "dd_rollout.cuh"

using namespace dd;

static_assert(DD_MIDDLE_SILU == MID_SILU && DD_MIDDLE_IDENTITY == MID_IDENTITY && DD_MIDDLE_RELU == MID_RELU &&
                  DD_MIDDLE_GELU == MID_GELU && DD_MIDDLE_GELU_TANH == MID_GELU_TANH && DD_MIDDLE_TANH == MID_TANH &&
                  DD_MIDDLE_SIGMOID == MID_SIGMOID && DD_MIDDLE_SILU_ROUNDED == MID_SILU_ROUNDED,
              "the header's middle kinds and the kernels' must agree");
static_assert(kMaxVerifyK1 == 64, "dd_verify_accept's position limit and its kernel's shared arrays must agree");

namespace {

typedef CUresult (*PFN_encodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                     const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                     CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

PFN_encodeTiled g_encode = nullptr;
std::once_flag g_encode_once;
char g_global_error[256] = "";

int round_up(int x, int m) { return (x + m - 1) / m * m; }
int ceil_div(long long x, long long m) { return (int)((x + m - 1) / m); }

}  // namespace

struct dd_handle {
  int device = 0;
  int num_sms = 0;
  dd_config cfg{};
  dd_weights w{};
  bool have_weights = false;
  int es = 2;   // bytes per activation / weight element: 2 (bf16, fp16) or 4 (fp32)
  int N1 = 16;  // MMA N of the h operand: batch rows padded to 16
  int N2 = 16;  // MMA N of the mid operand: 2 * batch (hi, lo) padded to 16
  int nslots = 0;
  void* zbuf = nullptr;       // [B * (p + S), E]
  void* midbuf = nullptr;     // [N2, E] rows 2b = hi, 2b+1 = lo, rest zero
  void* hbuf[2] = {nullptr, nullptr};  // [N1, G], rows >= B zero
  void* ghbuf = nullptr;      // [B, 3G]
  unsigned long long* slots = nullptr;  // [B, nslots]
  float* partials = nullptr;  // [2 * num_sms, 256, 128]
  unsigned int* counters = nullptr;
  int max_tiles = 0;
  int max_ctas = 0;
  unsigned int* status = nullptr;
  // Launch shape of the weight-streaming phases (tuning knobs, read from the
  // environment at dd_create: DD_RING_KB_BIG, DD_RING_KB_SMALL,
  // DD_MIN_SMEM_KB_BIG, DD_CTAS_PER_SM_BIG, DD_CTAS_PER_SM_SMALL).  "Big" phases stream the large
  // matrices (fc2, lm_head + W_z, the table); "small" ones W_s / W_hh.
  // Defaults measured on B200 (H = G = 4096, E = 12288, V = 151936): two
  // CTAs per SM with 72 KB rings (4 stages at batch <= 8) stream fc2 at
  // ~7.1 TB/s, and leave room on each SM for one CTA of the next phase, which
  // prefetches its weights under programmatic dependent launch; 100 KB rings
  // (no room) give ~6.5-6.9 TB/s and one CTA per SM ~5.5 TB/s at any depth.
  // More accumulators per slot and the packed weight layout measured no gain
  // at this shape, so both default off.
  int ring_kb_big = 72;
  int ring_kb_small = 72;
  int min_smem_kb_big = 0;
  int ctas_per_sm_big = 2;
  int ctas_per_sm_small = 2;
  int max_nacc = 1;               // DD_NACC
  int wide_two_per_sm = 1;        // DD_WIDE_TWO_PER_SM: passes of 64 < N <= 128 run two CTAs per SM
  int wide_epi_warps = 8;         // DD_WIDE_EPI_WARPS: epilogue warps of z / lm_head / table passes with N > 128
  int wide_pair = 0;              // DD_WIDE_PAIR: those passes as CTA pairs (M = 256 tiles, cta_group::2)
  int even_cut_pct = 60;          // DD_EVEN_CUT_PCT: slot fill from which weight streams cut tiles evenly
  int base_bufs = 0;              // DD_BASE_BUFS: fc2 base-logit buffers, 0 = by shared-memory room, 1 or 2
  int wide_one_slot = 0;          // DD_WIDE_ONE_SLOT: passes above N = 128 as two one-slot CTAs per SM
  int tmem_cols_per_cta = 128;    // DD_TMEM_COLS
  CUtensorMap tm_wz, tm_ws, tm_fc2, tm_whh, tm_lm, tm_mid, tm_h[2];
  // Vocab sharding (dd_set_vocab_shard): this rank owns vocab rows
  // [v_off, v_off + v_local) of fc2 / lm_head; world == 1 means unsharded.
  int v_off = 0;
  int v_local = 0;
  int world = 1;
  int rank = 0;
  unsigned long long* xbuf = nullptr;   // this rank's exchange buffer (also holds mid and gh)
  size_t xbuf_bytes = 0;
  size_t xsflag_off = 0, xmid_off = 0, xgh_off = 0;  // offsets inside xbuf (u64 units / bytes)
  unsigned int* xsdone = nullptr;       // per-slot finished-CTA counters of the s / gh phase
  // Sharded s / gh phase: rank j computes rows [e0[j], e1[j]) of W_s and
  // [g0[j], g1[j]) of W_hh (128-row aligned); off when a matrix has fewer
  // 128-row tiles than ranks.
  bool sgh_sharded = false;
  int e0[kMaxRanks] = {}, e1[kMaxRanks] = {}, g0[kMaxRanks] = {}, g1[kMaxRanks] = {};
  unsigned long long* xseq = nullptr;   // call sequence number (device)
  unsigned int* xdone = nullptr;        // per-slot finished-CTA counters
  unsigned long long* peer[kMaxRanks] = {};
  unsigned long long xtimeout_ns = 2000ull * 1000 * 1000;
  // Packed copies of the streamed weights (pack_tiles_kernel), made by
  // dd_set_weights unless the layout is set to row-major.
  bool pack = false;
  void* pk_wz = nullptr;
  void* pk_ws = nullptr;
  void* pk_fc2 = nullptr;
  void* pk_whh = nullptr;
  void* pk_lm = nullptr;
  // Persistent rollout (rollout_kernel): per-phase arrival counters + the
  // device-wide abort word; mode 0 = persistent when supported, 1 = phased
  // (default: measured faster on B200).
  unsigned int* rbar = nullptr;
  int rollout_mode = 1;
  int min_units_per_cta = 8;
  int l2_prefetch_kb = 0;  // DD_L2_PREFETCH_KB: weight bytes per CTA prefetched into L2 past the ring
  int l2_keep_mb = 0;      // DD_L2_KEEP_MB: s / gh weight bytes loaded evict_last, to stay in L2 across steps
  int middle = MID_SILU;    // dd_set_middle: the correction MLP's activation (and numerics)
  int fuse_cell = 0;
  int base_stage = 1;      // DD_BASE_STAGE: fc2 loads base-logit tiles by TMA at batch > 4       // DD_FUSE_CELL=1: the GRU cell runs in the fc2 launch's tail (measured slower: off)
  unsigned int* gbar = nullptr;  // grid barrier of the fused cell: [0] count, [1] generation
  // dd_verify_accept scratch: per-(row, position) argmax words + done counter
  static constexpr int kMaxVerifyPositions = 64;
  unsigned long long* vwords = nullptr;
  unsigned int* vdone = nullptr;
  int verify_per_sm[3] = {0, 0, 0};  // resident verify CTAs per SM, by logits dtype (f32, f16, bf16)
  // Opt-in state trace (dd_set_trace): per-step copies of z, h, gh and s.
  bool tracing = false;
  dd_trace trace{};
  // Opt-in per-launch timing (dd_set_timing): an event pair around each launch.
  static constexpr int kMaxTimed = 4096;
  bool timing = false;
  int n_timed = 0;
  int timed_kind[kMaxTimed];
  cudaEvent_t ev[2 * kMaxTimed] = {};
  char err[256] = "";
};

namespace {

int fail(dd_handle* h, int code, const char* fmt, ...) {
  char* dst = h ? h->err : g_global_error;
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(dst, 256, fmt, ap);
  va_end(ap);
  return code;
}

#define DD_CUDA(h, call)                                                                   \
  do {                                                                                     \
    cudaError_t e_ = (call);                                                               \
    if (e_ != cudaSuccess) return fail((h), DD_ECUDA, "%s: %s", #call, cudaGetErrorString(e_)); \
  } while (0)

int ensure_encoder(dd_handle* h) {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_encodeTiled>(fn);
  });
  if (!g_encode) return fail(h, DD_ECUDA, "cuTensorMapEncodeTiled is not available from the driver");
  return DD_OK;
}

// 2-D K-major tile map: rows of `k` elements (row stride `ld` elements),
// boxes of 64 x box_rows with 128-byte swizzle; out-of-range reads are zero.
int encode_kmajor(dd_handle* h, CUtensorMap* m, const void* ptr, int dtype, long long k, long long rows,
                  long long ld, int box_rows) {
  if (!ptr) return fail(h, DD_EINVAL, "null tensor pointer");
  if ((reinterpret_cast<uintptr_t>(ptr) & 15) != 0) return fail(h, DD_EINVAL, "tensor base is not 16-byte aligned");
  if ((ld * 2) % 16 != 0) return fail(h, DD_EINVAL, "row stride %lld elements is not a multiple of 16 bytes", ld);
  if (k <= 0 || rows <= 0 || ld < k) return fail(h, DD_EINVAL, "bad tensor shape k=%lld rows=%lld ld=%lld", k, rows, ld);
  if (box_rows < 1 || box_rows > 256) return fail(h, DD_EINVAL, "bad box rows %d", box_rows);
  int rc = ensure_encoder(h);
  if (rc) return rc;
  cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {(cuuint32_t)kChunkK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(m, dtype == DD_FP16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                        const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(h, DD_ECUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return DD_OK;
}

// 3-D map over base logits [B, rows_per_b, ld] (2-byte elements) with boxes of
// 128 columns x 1 position x B rows: one tile's base logits for one step.
int encode_base_map(dd_handle* h, CUtensorMap* m, const void* ptr, int dtype, long long ld, long long rows_per_b,
                    int batch) {
  int rc = ensure_encoder(h);
  if (rc) return rc;
  cuuint64_t dims[3] = {(cuuint64_t)ld, (cuuint64_t)rows_per_b, (cuuint64_t)batch};
  cuuint64_t strides[2] = {(cuuint64_t)(ld * 2), (cuuint64_t)(ld * rows_per_b * 2)};
  cuuint32_t box[3] = {(cuuint32_t)kTileM, 1u, (cuuint32_t)batch};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_encode(m, dtype == DD_FP16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3,
                        const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(h, DD_ECUDA, "cuTensorMapEncodeTiled (base logits) failed (%d)", (int)r);
  return DD_OK;
}

enum class PhaseClass { Big, Small };

int timing_begin(dd_handle* h, int kind, cudaStream_t st) {
  if (!h->timing) return DD_OK;
  if (h->n_timed >= dd_handle::kMaxTimed) return fail(h, DD_EINVAL, "timing record is full; call dd_read_timing");
  const int i = h->n_timed;
  for (int k = 0; k < 2; ++k)
    if (!h->ev[2 * i + k]) DD_CUDA(h, cudaEventCreate(&h->ev[2 * i + k]));
  h->timed_kind[i] = kind;
  DD_CUDA(h, cudaEventRecord(h->ev[2 * i], st));
  return DD_OK;
}

int timing_end(dd_handle* h, cudaStream_t st) {
  if (!h->timing) return DD_OK;
  DD_CUDA(h, cudaEventRecord(h->ev[2 * h->n_timed + 1], st));
  ++h->n_timed;
  return DD_OK;
}

// Opt the gemv kernel into the full 227 KB of dynamic shared memory, once
// per (device, element type).
template <typename T, int kPhase, int kEpiWarps = 4, bool kPair = false>
int set_kernel_attrs(dd_handle* h) {
  static bool done[64] = {};
  const int d = h->device & 63;
  if (!done[d]) {
    DD_CUDA(h, cudaFuncSetAttribute(gemv_stream_kernel<T, kPhase, kEpiWarps, kPair>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024));
    done[d] = true;
  }
  return DD_OK;
}

// Every launch carries programmatic stream serialisation, so it may start
// while the previous kernel on the stream drains (see griddepcontrol.* in
// the kernels).
struct Launch {
  cudaLaunchConfig_t cfg{};
  cudaLaunchAttribute attr[2];
  // cluster_x > 1: clusters of cluster_x CTAs along x (CTA pairs).
  Launch(dim3 grid, dim3 block, size_t smem, cudaStream_t st, unsigned cluster_x = 1) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cluster_x > 1) {
      attr[1].id = cudaLaunchAttributeClusterDimension;
      attr[1].val.clusterDim.x = cluster_x;
      attr[1].val.clusterDim.y = 1;
      attr[1].val.clusterDim.z = 1;
      cfg.numAttrs = 2;
    }
  }
};

// Whether a z / lm_head / table pass of N X rows runs as CTA pairs; its
// caller then encodes the X map with boxes of N / 2 rows (GemvParams::b_box_rows).
bool wide_pair_pass(const dd_handle* h, int n) {
  return h->wide_pair && h->wide_epi_warps == 8 && n > 128 && !h->pack;
}

// Fill the pass-independent launch fields of a gemv phase and launch it.
template <typename T, int kPhase>
int launch_gemv_tc(dd_handle* h, const CUtensorMap& a0, const CUtensorMap* a1, const CUtensorMap& b, GemvParams p,
                   PhaseClass cls, bool allow_split, cudaStream_t st) {
  p.KC = ceil_div(p.K, kChunkK);
  int tiles = 0;
  for (int s = 0; s < p.nseg; ++s) {
    p.seg[s].tiles = ceil_div(p.seg[s].rows, kTileM);
    tiles += p.seg[s].tiles;
  }
  if (tiles > h->max_tiles) return fail(h, DD_EINVAL, "phase has %d tiles > %d", tiles, h->max_tiles);
  constexpr bool kXRowMajor = kPhase == PH_ZLM || kPhase == PH_Z || kPhase == PH_TABLE;
  // CTA pairs: the caller encoded the X map with half-height boxes.
  const bool pair = kXRowMajor && p.b_box_rows > 0 && 2 * p.b_box_rows == p.N && wide_pair_pass(h, p.N) &&
                    !p.packed[0] && !p.packed[1];
  if (!pair) {
    // A half-height X map only makes sense for a pair launch: its loads would
    // deliver half the bytes a lone CTA's stage waits for.
    if (p.b_box_rows > 0 && p.b_box_rows != p.N)
      return fail(h, DD_EINVAL, "X map with %d-row boxes for a %d-row pass without CTA pairs", p.b_box_rows, p.N);
    p.b_box_rows = p.N;
  }
  p.tiles128 = tiles;
  p.units = (long long)(pair ? (tiles + 1) / 2 : tiles) * p.KC;
  p.b_bytes = (uint32_t)p.b_box_rows * 128u;
  p.stage_bytes = kATileBytes + p.b_bytes;
  // Wide passes (N > 64) take one CTA per SM with a 196 KB ring, except that
  // up to N = 128 three stages of at most 32 KB and 2 x 128 TMEM columns
  // leave room for a second CTA on the SM.  Narrower passes: the class ring.
  const bool wide2 = p.N > 64 && p.N <= 128 && h->wide_two_per_sm;
  // Above N = 128, optionally two CTAs per SM with one accumulator slot and
  // two stages each (2 x 256 TMEM columns per SM): each CTA's epilogue
  // overlaps the other's MMAs instead of its own.
  const bool wide1 = kXRowMajor && p.N > 128 && !pair && h->wide_one_slot;
  uint32_t ring_budget =
      p.N > 64 ? (wide2 ? 3u * p.stage_bytes : wide1 ? 2u * p.stage_bytes : 196u * 1024u)
               : (uint32_t)(cls == PhaseClass::Big ? h->ring_kb_big : h->ring_kb_small) * 1024u;
  // fc2 with base-logit staging: four stages whenever two CTAs with four
  // still fit on an SM (batch 9-24: 20-22 KB stages, 80-88 KB, past the 72 KB
  // ring budget; at batch 16, E = 12288 fc2 584 -> 568 us).  Above batch 24
  // two CTAs with four stages fit only with one base buffer, which the
  // producer then fills between stages.
  p.base_bufs = 2;
  if (cls == PhaseClass::Big && p.N <= 64 && p.base_stage_bytes) {
    auto fits4 = [&](int nb) {
      return 2u * (4u * p.stage_bytes + 1024u + kSmemTail + (uint32_t)nb * p.base_stage_bytes + 1024u) <= 228u * 1024u;
    };
    p.base_bufs = h->base_bufs ? h->base_bufs : (fits4(2) ? 2 : (fits4(1) ? 1 : 2));
    if (fits4(p.base_bufs) && ring_budget < 4u * p.stage_bytes) ring_budget = 4u * p.stage_bytes;
  }
  // At least four stages; three when the base-logit buffers take the room of
  // the fourth (fc2 above batch 8, whose stages outgrow 18 KB) or for the
  // two-per-SM wide passes, so that two CTAs still share an SM.
  p.stages = wide1 ? 2
                   : std::max(p.base_stage_bytes || wide2 ? 3 : 4,
                              std::min<int>(kMaxStages, (int)(ring_budget / p.stage_bytes)));
  p.l2_prefetch_units = pair ? 0 : (int)((long long)h->l2_prefetch_kb * 1024 / kATileBytes);
  // The s / gh weights (read once per step, ~109 MB at E = 1024) can stay in
  // the 126 MB L2 from one step to the next while fc2 streams past them
  // evict_first: segments that fit the budget, W_hh first, load evict_last.
  p.w_keep[0] = p.w_keep[1] = 0;
  if constexpr (kPhase == PH_SGH || kPhase == PH_GH) {
    long long left = (long long)h->l2_keep_mb << 20;
    for (int s = p.nseg - 1; s >= 0; --s) {
      const long long bytes = (long long)p.seg[s].rows * p.K * (long long)sizeof(T);
      if (bytes <= left) {
        p.w_keep[s] = 1;
        left -= bytes;
      }
    }
  }
  // X-row-major outputs (z, base logits, the table): a staging area per
  // epilogue warpgroup; passes wider than 128 columns (one CTA per SM) get two
  // warpgroups.
  const bool epi8 = kXRowMajor && p.N > 128 && h->wide_epi_warps == 8 && !wide1;
  p.xpose_bytes = kXRowMajor ? (epi8 ? 2u : 1u) * kXposeBytes : 0u;
  const uint32_t fixed = 1024 + kSmemTail + p.xpose_bytes + (uint32_t)p.base_bufs * p.base_stage_bytes;
  if ((size_t)p.stages * p.stage_bytes + fixed > 227 * 1024) p.stages = (227 * 1024 - fixed) / p.stage_bytes;
  p.acc_slots = wide1 ? 1 : 2;  // the epilogue of one tile overlaps the next tile's MMAs (2 x 256 columns at most)
  // Up to four accumulators per slot within the per-CTA TMEM budget, so that
  // co-resident CTAs (2 per SM plus the next phase's) never wait for TMEM.
  p.nacc = 1;
  while (p.nacc < h->max_nacc && p.acc_slots * p.nacc * 2 * p.N <= h->tmem_cols_per_cta) p.nacc *= 2;
  uint32_t cols = 32;
  while (cols < (uint32_t)(p.acc_slots * p.nacc * p.N)) cols <<= 1;
  p.tmem_cols = cols;
  p.idesc = pair ? idesc_f16_m256((uint32_t)p.N, std::is_same<T, __half>::value ? 0u : 1u)
               : idesc_f16((uint32_t)p.N, std::is_same<T, __half>::value ? 0u : 1u);
  p.partials = h->partials;
  p.tile_counters = h->counters;
  p.status = h->status;
  size_t smem = (size_t)p.stages * p.stage_bytes + fixed;
  // Big phases reserve enough shared memory that two CTAs of the same phase
  // never share an SM, while one small-phase CTA still fits beside them.
  if (cls == PhaseClass::Big && smem < (size_t)h->min_smem_kb_big * 1024) smem = (size_t)h->min_smem_kb_big * 1024;
  if (smem > 227 * 1024) return fail(h, DD_EINVAL, "shared memory %zu exceeds 227 KB", smem);
  // One wave: no more CTAs than fit on the SMs at once (the stream-K split
  // gives each the same work; a second wave would only add a tail).
  const int fit = (int)(228u * 1024u / (uint32_t)(smem + 1024));
  const int per_sm = std::max(1, std::min(fit, cls == PhaseClass::Big ? h->ctas_per_sm_big : h->ctas_per_sm_small));
  // At least min_units_per_cta units per CTA: a tile split over more CTAs
  // costs its finisher one partial per CTA to add, more than the stream time
  // the extra CTAs would save.
  const long long slots = (long long)h->num_sms * per_sm;
  int grid = (int)std::min<long long>(slots, allow_split ? std::max<long long>(1, p.units / h->min_units_per_cta) : tiles);
  // Weight streams (N <= 64) with no more tiles than slots: every tile is cut
  // into the same number k <= 4 of CTA ranges (k = 1: one whole tile per CTA),
  // as long as that fills a clear majority of the slots (even_cut_pct, 60 %).
  // A finisher then adds at most k - 1 partials, where a stream-K cut over all
  // slots can leave it a longer chain than the extra slots save (s / gh at
  // E = 12288: 192 tiles, k = 1; at E = 1024: 104 tiles, k = 2).  Near half the
  // slots the cut leaves about one CTA per SM, which streams at the one-CTA
  // rate (~5.3 TB/s): fc2 of an 8-way vocab shard (149 tiles) took 148 µs that
  // way against 127 µs over all slots.  Wider passes are closer to
  // tensor-bound and keep every SM.
  if (allow_split && p.N <= 64 && tiles <= slots) {
    const long long k = std::min<long long>(4, slots / tiles);
    if (100LL * tiles * k >= (long long)h->even_cut_pct * slots) grid = (int)(tiles * k);
  }
  if (grid < 1) grid = 1;
  int rc = DD_OK;
  if constexpr (kXRowMajor) {
    if (pair) {  // clusters of 2 on the pair-tile partition
      const long long pair_slots = (long long)h->num_sms / 2;
      const long long pairs = std::max<long long>(
          1, std::min<long long>(pair_slots, allow_split ? p.units / h->min_units_per_cta : (tiles + 1) / 2));
      rc = set_kernel_attrs<T, kPhase, 8, true>(h);
      if (rc) return rc;
      rc = timing_begin(h, kPhase, st);
      if (rc) return rc;
      Launch L(dim3((unsigned)(2 * pairs)), dim3((kEpiWarp0 + 8) * 32), smem, st, 2);
      DD_CUDA(h, cudaLaunchKernelEx(&L.cfg, gemv_stream_kernel<T, kPhase, 8, true>, a0, a1 ? *a1 : a0, b, p));
      return timing_end(h, st);
    }
    if (epi8) {
      rc = set_kernel_attrs<T, kPhase, 8>(h);
      if (rc) return rc;
      rc = timing_begin(h, kPhase, st);
      if (rc) return rc;
      Launch L(dim3(grid), dim3((kEpiWarp0 + 8) * 32), smem, st);
      DD_CUDA(h, cudaLaunchKernelEx(&L.cfg, gemv_stream_kernel<T, kPhase, 8>, a0, a1 ? *a1 : a0, b, p));
      return timing_end(h, st);
    }
  }
  rc = set_kernel_attrs<T, kPhase>(h);
  if (rc) return rc;
  rc = timing_begin(h, kPhase, st);
  if (rc) return rc;
  Launch L(dim3(grid), dim3(kThreads), smem, st);
  DD_CUDA(h, cudaLaunchKernelEx(&L.cfg, gemv_stream_kernel<T, kPhase>, a0, a1 ? *a1 : a0, b, p));
  return timing_end(h, st);
}

// fp32 heads: the phase's rows through gemv_f32_kernel, in launches of at
// most kF32MaxN X rows (the weights are read once per launch).
template <int kPhase>
int launch_gemv_f32(dd_handle* h, GemvParams p, cudaStream_t st) {
  int rows = 0;
  for (int s = 0; s < p.nseg; ++s) rows += p.seg[s].rows;
  p.status = h->status;
  const int n_begin = p.n_off;
  const int n_total = kPhase == PH_FC2 ? p.B : p.n_valid;
  const int grid = std::max(1, ceil_div(rows, kF32RowsPerCta));
  for (int n0 = 0; n0 < n_total; n0 += kF32MaxN) {
    p.n_off = n_begin + n0;
    p.n_valid = std::min(kF32MaxN, n_total - n0);
    int rc = timing_begin(h, kPhase, st);
    if (rc) return rc;
    Launch L(dim3(grid), dim3(kF32Threads), 0, st);
    DD_CUDA(h, cudaLaunchKernelEx(&L.cfg, gemv_f32_kernel<kPhase>, p));
    rc = timing_end(h, st);
    if (rc) return rc;
  }
  return DD_OK;
}

// One contraction phase: tcgen05 weight streaming for bf16 / fp16 heads,
// CUDA-core fp32 FMA for fp32 heads.
template <typename T, int kPhase>
int launch_gemv(dd_handle* h, const CUtensorMap& a0, const CUtensorMap* a1, const CUtensorMap& b, GemvParams p,
                PhaseClass cls, bool allow_split, cudaStream_t st) {
  if constexpr (std::is_same<T, float>::value)
    return launch_gemv_f32<kPhase>(h, p, st);
  else
    return launch_gemv_tc<T, kPhase>(h, a0, a1, b, p, cls, allow_split, st);
}

Exchange make_exchange(const dd_handle* h);

// The handle-wide fields of a GRU step.
void fill_cell(const dd_handle* h, CellParams& cp) {
  cp.B = h->cfg.batch;
  cp.G = h->cfg.gru_hidden;
  cp.V = h->cfg.vocab;
  cp.table = h->w.table;
  cp.table_ld = h->w.table_ld;
  cp.b_hh = h->w.b_hh;
  cp.status = h->status;
  cp.xchg = make_exchange(h);
  cp.xbuf = h->xbuf;
}

template <typename T>
int launch_cell(dd_handle* h, CellParams cp, cudaStream_t st) {
  fill_cell(h, cp);
  const int threads = cp.B * (cp.G / 8);
  int rc = timing_begin(h, DD_PHASE_CELL, st);
  if (rc) return rc;
  Launch L(dim3(ceil_div(threads, 128)), dim3(128), 0, st);
  DD_CUDA(h, cudaLaunchKernelEx(&L.cfg, cell_kernel<T>, cp));
  return timing_end(h, st);
}

Exchange make_exchange(const dd_handle* h) {
  Exchange x;
  memset(&x, 0, sizeof(x));
  x.world = h->world;
  x.rank = h->rank;
  for (int j = 0; j < h->world; ++j) x.peer[j] = h->peer[j];
  x.seq = h->xseq;
  x.done = h->xdone;
  x.nslots = h->nslots;
  x.B = h->cfg.batch;
  x.timeout_ns = h->xtimeout_ns;
  x.sflag_off = h->xsflag_off;
  x.mid_off = h->xmid_off;
  x.gh_off = h->xgh_off;
  x.sdone = h->xsdone;
  return x;
}

GemvParams base_params(const dd_handle* h) {
  GemvParams p;
  memset(&p, 0, sizeof(p));
  p.B = h->cfg.batch;
  p.V = h->v_local;
  p.E = h->cfg.emb_dim;
  p.G3 = 3 * h->cfg.gru_hidden;
  p.slots = h->slots;
  p.nslots = h->nslots;
  p.v_off = h->v_off;
  p.base_ld = h->cfg.vocab;
  p.base_out_ld = h->v_local;
  p.base_voff = h->v_off;
  p.xchg = make_exchange(h);
  p.sflag_slot = -1;
  p.middle = h->middle;
  return p;
}

__global__ void bump_sequence_kernel(unsigned long long* seq) {
  pdl_launch_dependents();
  pdl_wait_primary();
  *seq += 1ull;
}

// Start of a call on a vocab-sharded handle: a new sequence number, so that
// the exchange flags of this call differ from every earlier call's.
int begin_exchange(dd_handle* h, cudaStream_t st) {
  if (h->world <= 1) return DD_OK;
  DD_CUDA(h, cudaMemsetAsync(h->xdone, 0, (size_t)h->nslots * 4, st));
  DD_CUDA(h, cudaMemsetAsync(h->xsdone, 0, (size_t)h->nslots * 4, st));
  Launch L(dim3(1), dim3(1), 0, st);
  DD_CUDA(h, cudaLaunchKernelEx(&L.cfg, bump_sequence_kernel, h->xseq));
  return DD_OK;
}

// Sharded s / gh phase: copy the other ranks' mid / gh slices of `slot` here.
int launch_gather(dd_handle* h, int slot, bool with_gh, cudaStream_t st) {
  GatherParams gp;
  memset(&gp, 0, sizeof(gp));
  gp.xchg = make_exchange(h);
  gp.xbuf = h->xbuf;
  gp.slot = slot;
  gp.mid_rows = 2 * h->cfg.batch;
  gp.E = h->cfg.emb_dim;
  gp.G3 = 3 * h->cfg.gru_hidden;
  gp.B = h->cfg.batch;
  long long vecs = 0;
  for (int j = 0; j < h->world; ++j) {
    gp.e0[j] = h->e0[j];
    gp.e1[j] = h->e1[j];
    gp.g0[j] = h->g0[j];
    gp.g1[j] = h->g1[j];
    if (j != h->rank)
      vecs += (long long)gp.mid_rows * (h->e1[j] - h->e0[j]) / 8 +
              (with_gh ? (long long)gp.B * (h->g1[j] - h->g0[j]) / 8 : 0);
  }
  gp.with_gh = with_gh ? 1 : 0;
  gp.status = h->status;
  const int grid = (int)std::max<long long>(1, std::min<long long>(2LL * h->num_sms, (vecs + 255) / 256));
  int rc = timing_begin(h, DD_PHASE_GATHER, st);
  if (rc) return rc;
  Launch L(dim3(grid), dim3(256), 0, st);
  DD_CUDA(h, cudaLaunchKernelEx(&L.cfg, gather_slices_kernel, gp));
  return timing_end(h, st);
}

// Trace copies (dd_set_trace): `rows` x `cols` elements of the weight dtype
// from a scratch buffer into entry `idx` of a caller trace array.
int trace_copy(dd_handle* h, void* dst, int idx, const void* src, long long rows, long long cols, cudaStream_t st) {
  if (!h->tracing || !dst) return DD_OK;
  const size_t bytes = (size_t)rows * cols * h->es;
  DD_CUDA(h, cudaMemcpyAsync(static_cast<uint8_t*>(dst) + (size_t)idx * bytes, src, bytes, cudaMemcpyDeviceToDevice, st));
  return DD_OK;
}

// Z (+ lm_head) phase over the X = parallel_hiddens rows, in passes of <= 256 rows.
template <typename T>
int run_z_phase(dd_handle* h, const void* ph, int positions, int npre, void* base_out, cudaStream_t st) {
  const dd_config& c = h->cfg;
  const int rows = c.batch * positions;
  CUtensorMap tm_x;
  // Passes of at most 256 X rows (one MMA's N), as equal as the 16-row MMA
  // granularity allows: 480 rows as 2 x 240, 272 as 2 x 144 (not 256 + 16,
  // whose second pass would stream every weight for 16 rows).
  const int passes = ceil_div(rows, 256);
  const int n_pass = round_up(ceil_div(rows, passes), 16);
  const int x_box = wide_pair_pass(h, n_pass) ? n_pass / 2 : n_pass;  // CTA pairs load half the rows each
  int rc = DD_OK;
  if constexpr (!std::is_same<T, float>::value) {
    rc = encode_kmajor(h, &tm_x, ph, c.dtype, c.hidden, rows, c.hidden, x_box);
    if (rc) return rc;
  }
  for (int n_off = 0; n_off < rows; n_off += n_pass) {
    GemvParams p = base_params(h);
    p.x32 = static_cast<const float*>(ph);
    p.x32_ld = c.hidden;
    p.w32[0] = static_cast<const float*>(base_out ? h->w.lm_head : h->w.fc1);
    p.w32_ld[0] = base_out ? h->w.lm_head_ld : h->w.fc1_ld;
    p.w32[1] = static_cast<const float*>(h->w.fc1);
    p.w32_ld[1] = h->w.fc1_ld;
    const int n_valid = std::min(n_pass, rows - n_off);
    p.N = n_pass;  // the TMA box height (x_box: N, or N / 2 per CTA of a pair), so expect_tx matches the loads
    p.b_box_rows = x_box;
    p.n_off = n_off;
    p.n_valid = n_valid;
    p.K = c.hidden;
    p.z_out = h->zbuf;
    p.fc1_bias = h->w.fc1_bias;
    if (base_out) {
      p.nseg = 2;
      p.seg[0] = {h->v_local, 0, EPI_LMHEAD};
      if (npre > 0 && n_off + n_pass >= rows) {  // last pass: the prefix argmax words are final
        p.xslot0 = 0;
        p.xslot1 = npre;
      }
      p.seg[1] = {c.emb_dim, 0, EPI_ZPROJ};
      p.base_out = base_out;
      p.kpos = positions;
      p.npre = npre;
      p.packed[0] = static_cast<const uint8_t*>(h->pk_lm);
      p.packed[1] = static_cast<const uint8_t*>(h->pk_wz);
      rc = launch_gemv<T, PH_ZLM>(h, h->tm_lm, &h->tm_wz, tm_x, p, PhaseClass::Big, true, st);
    } else {
      p.nseg = 1;
      p.seg[0] = {c.emb_dim, 0, EPI_ZPROJ};
      p.packed[0] = static_cast<const uint8_t*>(h->pk_wz);
      rc = launch_gemv<T, PH_Z>(h, h->tm_wz, nullptr, tm_x, p, PhaseClass::Big, true, st);
    }
    if (rc) return rc;
  }
  return trace_copy(h, h->trace.z, 0, h->zbuf, rows, c.emb_dim, st);
}

// GRU prefix + S rollout steps.  Token sources: ids (runner) or the prefix
// argmax words (draft block); outputs to out[b * out_ld + out_col0 + t].
template <typename T>
int run_rollout(dd_handle* h, const int64_t* ids, int ids_ld, int n_prefix_ids, int npre, int positions,
                const void* base, long long base_ld, long long base_voff, int64_t* out, int out_ld, int out_col0,
                int64_t* prefix_out, cudaStream_t st) {
  const dd_config& c = h->cfg;
  int rc;
  int cur = 0;
  // fc2 at more than four batch rows: each tile's base logits arrive by TMA
  // (16-byte row strides and column offset needed; 2-byte types only).
  CUtensorMap tm_base;
  uint32_t base_stage = 0;
  if constexpr (!std::is_same<T, float>::value) {
    if (c.batch > 4 && h->base_stage && (base_ld % 8) == 0 && (base_voff % 8) == 0 &&
        (reinterpret_cast<uintptr_t>(base) & 15) == 0) {
      rc = encode_base_map(h, &tm_base, base, c.dtype, base_ld, positions, c.batch);
      if (rc) return rc;
      base_stage = (uint32_t)c.batch * kTileM * 2;
    }
  }
  // h0 from the first prefix token, zero state.
  {
    CellParams cp;
    memset(&cp, 0, sizeof(cp));
    cp.src = 0;
    cp.ids = ids;
    cp.ids_ld = ids_ld;
    cp.ids_col = 0;
    cp.out = prefix_out;
    cp.out_ld = out_ld;
    cp.out_col = 0;
    cp.h_zero = 1;
    cp.write_h = 1;
    cp.h_out = h->hbuf[0];
    rc = launch_cell<T>(h, cp, st);
    if (!rc) rc = trace_copy(h, h->trace.h, 0, h->hbuf[0], c.batch, c.gru_hidden, st);
    if (rc) return rc;
  }
  const int n_prefix_total = n_prefix_ids + npre;  // GRU inputs before the rollout
  for (int j = 1; j < n_prefix_total; ++j) {
    GemvParams p = base_params(h);
    p.nseg = 1;
    p.seg[0] = {3 * c.gru_hidden, 0, EPI_GH};
    p.K = c.gru_hidden;
    p.N = h->N1;
    p.n_valid = c.batch;
    p.gh_out = h->ghbuf;
    p.b_hh = h->w.b_hh;
    p.packed[0] = static_cast<const uint8_t*>(h->pk_whh);
    p.w32[0] = static_cast<const float*>(h->w.w_hh);
    p.w32_ld[0] = h->w.w_hh_ld;
    p.x32 = static_cast<const float*>(h->hbuf[cur]);
    p.x32_ld = c.gru_hidden;
    rc = launch_gemv<T, PH_GH>(h, h->tm_whh, nullptr, h->tm_h[cur], p, PhaseClass::Small, true, st);
    if (!rc) rc = trace_copy(h, h->trace.gh, j - 1, h->ghbuf, c.batch, 3LL * c.gru_hidden, st);
    if (rc) return rc;
    CellParams cp;
    memset(&cp, 0, sizeof(cp));
    if (j < n_prefix_ids) {
      cp.src = 0;
      cp.ids = ids;
      cp.ids_ld = ids_ld;
      cp.ids_col = j;
    } else {
      cp.src = 1;
      cp.slots = h->slots;
      cp.nslots = h->nslots;
      cp.slot_idx = j - n_prefix_ids;
      cp.out = prefix_out;
      cp.out_ld = out_ld;
      cp.out_col = j;
    }
    cp.write_h = 1;
    cp.gh = h->ghbuf;
    cp.h_in = h->hbuf[cur];
    cp.h_out = h->hbuf[cur ^ 1];
    rc = launch_cell<T>(h, cp, st);
    if (!rc) rc = trace_copy(h, h->trace.h, j, h->hbuf[cur ^ 1], c.batch, c.gru_hidden, st);
    if (rc) return rc;
    cur ^= 1;
  }
  for (int t = 0; t < c.steps; ++t) {
    const bool last = t + 1 == c.steps;
    {
      GemvParams p = base_params(h);
      p.nseg = last ? 1 : 2;
      p.seg[0] = {c.emb_dim, 0, EPI_SPROJ_MID, 0};
      p.seg[1] = {3 * c.gru_hidden, 0, EPI_GH, 0};
      if (h->sgh_sharded) {
        const int r = h->rank;
        p.seg[0] = {h->e1[r] - h->e0[r], 0, EPI_SPROJ_MID, h->e0[r]};
        p.seg[1] = {h->g1[r] - h->g0[r], 0, EPI_GH, h->g0[r]};
        p.sflag_slot = npre + t;
      }
      p.K = c.gru_hidden;
      p.N = h->N1;
      p.n_valid = c.batch;
      p.t = t;
      p.z_src = h->zbuf;
      p.z_rows_per_b = positions;
      p.z_pos_off = npre;
      p.mid_out = h->midbuf;
      p.gh_out = h->ghbuf;
      p.b_hh = h->w.b_hh;
      if (h->tracing && h->trace.s)
        p.s_out = static_cast<uint8_t*>(h->trace.s) + (size_t)t * c.batch * c.emb_dim * h->es;
      p.packed[0] = static_cast<const uint8_t*>(h->pk_ws);
      p.packed[1] = static_cast<const uint8_t*>(h->pk_whh);
      p.w32[0] = static_cast<const float*>(h->w.fc1) + c.hidden;  // W_s = fc1[:, H:]
      p.w32_ld[0] = h->w.fc1_ld;
      p.w32[1] = static_cast<const float*>(h->w.w_hh);
      p.w32_ld[1] = h->w.w_hh_ld;
      p.x32 = static_cast<const float*>(h->hbuf[cur]);
      p.x32_ld = c.gru_hidden;
      rc = launch_gemv<T, PH_SGH>(h, h->tm_ws, last ? nullptr : &h->tm_whh, h->tm_h[cur], p, PhaseClass::Small, true, st);
      if (!rc && !last)
        rc = trace_copy(h, h->trace.gh, n_prefix_total - 1 + t, h->ghbuf, c.batch, 3LL * c.gru_hidden, st);
      if (rc) return rc;
      if (h->sgh_sharded) {
        rc = launch_gather(h, npre + t, !last, st);
        if (rc) return rc;
      }
    }
    {
      GemvParams p = base_params(h);
      p.nseg = 1;
      p.seg[0] = {h->v_local, 0, EPI_FC2_ARGMAX};
      p.K = c.emb_dim;
      p.N = h->N2;
      p.n_valid = 2 * c.batch;
      p.t = t;
      p.npre = npre;
      p.base_src = base;
      p.base_ld = base_ld;
      p.base_voff = base_voff;
      p.xslot0 = npre + t;
      p.xslot1 = npre + t + 1;
      p.packed[0] = static_cast<const uint8_t*>(h->pk_fc2);
      p.base_rows_per_b = positions;
      p.base_pos_off = npre;
      p.fc2_bias = h->w.fc2_bias;
      p.w32[0] = static_cast<const float*>(h->w.fc2);
      p.w32_ld[0] = h->w.fc2_ld;
      p.x32 = static_cast<const float*>(h->midbuf);  // fp32 heads: mid is [B, E] fp32
      p.x32_ld = c.emb_dim;
      CellParams cp;
      memset(&cp, 0, sizeof(cp));
      cp.src = 1;
      cp.slots = h->slots;
      cp.nslots = h->nslots;
      cp.slot_idx = npre + t;
      cp.out = out;
      cp.out_ld = out_ld;
      cp.out_col = out_col0 + t;
      cp.write_h = last ? 0 : 1;
      cp.torch_cell = h->middle != MID_SILU;  // the PyTorch branch's cell (the prefix GRU is nn.GRU in both)
      cp.gh = h->ghbuf;
      cp.h_in = h->hbuf[cur];
      cp.h_out = h->hbuf[cur ^ 1];
      // The step's GRU cell runs in the fc2 launch itself (after a grid-wide
      // barrier) on unsharded bf16 / fp16 handles; a launch of its own otherwise.
      const bool fuse = h->fuse_cell && h->world == 1 && !h->tracing && !std::is_same<T, float>::value;
      if (fuse) {
        fill_cell(h, cp);
        p.fused_cell = 1;
        p.gbar = h->gbar;
        p.cell = cp;
      }
      p.base_stage_bytes = base_stage;
      rc = launch_gemv<T, PH_FC2>(h, h->tm_fc2, base_stage ? &tm_base : nullptr, h->tm_mid, p, PhaseClass::Big, true,
                                  st);
      if (!rc && !fuse) rc = launch_cell<T>(h, cp, st);
      if (!rc && !last) rc = trace_copy(h, h->trace.h, n_prefix_total + t, h->hbuf[cur ^ 1], c.batch, c.gru_hidden, st);
      if (rc) return rc;
      cur ^= 1;
    }
  }
  return DD_OK;
}

// The rollout as one persistent cooperative kernel (dd_rollout.cuh); the same
// phases, in the same order, as run_rollout launches one by one.  Returns
// DD_EUNSUPPORTED (and launches nothing) when the handle or the shapes need
// the phased path: vocab sharding, more phases than the table holds, or a
// device that cannot keep every CTA resident.
template <typename T>
int run_rollout_persistent(dd_handle* h, const int64_t* ids, int ids_ld, int n_prefix_ids, int npre, int positions,
                           const void* base, long long base_ld, long long base_voff, int64_t* out, int out_ld,
                           int out_col0, int64_t* prefix_out, cudaStream_t st) {
  const dd_config& c = h->cfg;
  const int n_prefix_total = n_prefix_ids + npre;
  const int nphases = 1 + 2 * (n_prefix_total - 1) + 3 * c.steps;
  if (h->rollout_mode != 0 || h->world > 1 || h->tracing || h->middle != MID_SILU || nphases > kMaxRollPhases)
    return DD_EUNSUPPORTED;
  static RollParams rp;  // ~10 KB: kept off the stack; the handle is not thread-safe anyway
  memset(&rp, 0, sizeof(rp));
  GemvParams& gp = rp.gp;
  gp = base_params(h);
  gp.npre = npre;
  gp.base_src = base;
  gp.base_rows_per_b = positions;
  gp.base_pos_off = npre;
  gp.base_ld = base_ld;
  gp.base_voff = base_voff;
  gp.fc2_bias = h->w.fc2_bias;
  gp.z_src = h->zbuf;
  gp.z_rows_per_b = positions;
  gp.z_pos_off = npre;
  gp.mid_out = h->midbuf;
  gp.gh_out = h->ghbuf;
  gp.b_hh = h->w.b_hh;
  gp.partials = h->partials;
  gp.tile_counters = h->counters;
  gp.status = h->status;
  gp.acc_slots = 2;
  gp.nacc = 1;
  CellParams& cp = rp.cp;
  cp.B = c.batch;
  cp.G = c.gru_hidden;
  cp.V = c.vocab;
  cp.ids = ids;
  cp.ids_ld = ids_ld;
  cp.slots = h->slots;
  cp.nslots = h->nslots;
  cp.out = out;
  cp.out_ld = out_ld;
  cp.table = h->w.table;
  cp.table_ld = h->w.table_ld;
  cp.gh = h->ghbuf;
  cp.b_hh = h->w.b_hh;
  cp.status = h->status;
  rp.hbuf[0] = h->hbuf[0];
  rp.hbuf[1] = h->hbuf[1];
  rp.bar = h->rbar;
  rp.abort_word = h->rbar + kMaxRollPhases;
  rp.ab_fmt = c.dtype == DD_FP16 ? 0u : 1u;
  const int G3 = 3 * c.gru_hidden;
  auto gemv = [&](RollPhase& P, int nseg, GemvSeg s0, GemvSeg s1, int a0, int a1, int bmap, int K, int N, int nv,
                  int t) {
    P.type = RP_GEMV;
    P.nseg = nseg;
    s0.tiles = ceil_div(s0.rows, kTileM);
    s1.tiles = nseg > 1 ? ceil_div(s1.rows, kTileM) : 0;
    P.seg[0] = s0;
    P.seg[1] = s1;
    P.a_map[0] = a0;
    P.a_map[1] = a1;
    P.b_map = bmap;
    P.K = K;
    P.KC = ceil_div(K, kChunkK);
    P.N = N;
    P.n_valid = nv;
    P.t = t;
  };
  // Prefix tokens are written only by dd_draft_block, into the same array.
  if (prefix_out != nullptr && prefix_out != out) return DD_EUNSUPPORTED;
  const bool prefix_writes_out = prefix_out != nullptr;
  int n = 0, cur = 0;
  {
    RollPhase& P = rp.ph[n++];
    P.type = RP_CELL;
    P.src = 0;
    P.ids_col = 0;
    P.out_col = prefix_writes_out ? 0 : -1;
    P.h_zero = 1;
    P.write_h = 1;
    P.h_out = 0;
  }
  for (int j = 1; j < n_prefix_total; ++j) {
    gemv(rp.ph[n++], 1, GemvSeg{G3, 0, EPI_GH, 0}, GemvSeg{0, 0, 0, 0}, 1, 1, cur, c.gru_hidden, h->N1, c.batch, 0);
    RollPhase& P = rp.ph[n++];
    P.type = RP_CELL;
    if (j < n_prefix_ids) {
      P.src = 0;
      P.ids_col = j;
      P.out_col = -1;
    } else {
      P.src = 1;
      P.slot_idx = j - n_prefix_ids;
      P.out_col = prefix_writes_out ? j : -1;
    }
    P.write_h = 1;
    P.h_in = cur;
    P.h_out = cur ^ 1;
    cur ^= 1;
  }
  for (int t = 0; t < c.steps; ++t) {
    const bool last = t + 1 == c.steps;
    gemv(rp.ph[n++], last ? 1 : 2, GemvSeg{c.emb_dim, 0, EPI_SPROJ_MID, 0}, GemvSeg{G3, 0, EPI_GH, 0}, 0, 1, cur,
         c.gru_hidden, h->N1, c.batch, t);
    gemv(rp.ph[n++], 1, GemvSeg{h->v_local, 0, EPI_FC2_ARGMAX, 0}, GemvSeg{0, 0, 0, 0}, 2, 2, 2, c.emb_dim, h->N2,
         2 * c.batch, t);
    RollPhase& P = rp.ph[n++];
    P.type = RP_CELL;
    P.src = 1;
    P.slot_idx = npre + t;
    P.out_col = out_col0 + t;
    P.write_h = last ? 0 : 1;
    P.h_in = cur;
    P.h_out = cur ^ 1;
    cur ^= 1;
  }
  rp.nphases = n;
  int tiles_max = 0;
  for (int i = 0; i < n; ++i)
    if (rp.ph[i].type == RP_GEMV) tiles_max = std::max(tiles_max, rp.ph[i].seg[0].tiles + rp.ph[i].seg[1].tiles);
  if (tiles_max > h->max_tiles) return fail(h, DD_EINVAL, "rollout phase has %d tiles > %d", tiles_max, h->max_tiles);
  // Launch shape: one CTA per SM holding ctas_per_sm_big pipelines, each with
  // one ring layout sized for the wider activation operand.
  rp.subs = h->ctas_per_sm_big;
  rp.n_max = std::max(h->N1, h->N2);
  rp.stage_bytes = kATileBytes + (uint32_t)rp.n_max * 128u;
  rp.stages = std::max(4, std::min<int>(kMaxStages, (int)((uint32_t)h->ring_kb_big * 1024u / rp.stage_bytes)));
  const int fit = (int)(((227u * 1024u - 1024u) / (uint32_t)rp.subs - kSmemTail) / rp.stage_bytes);
  rp.stages = std::min(rp.stages, fit);
  if (rp.stages < 2) return DD_EUNSUPPORTED;
  uint32_t cols = 32;
  while (cols < (uint32_t)(2 * rp.n_max)) cols <<= 1;
  rp.tmem_cols = cols;
  const size_t smem = 1024 + (size_t)rp.subs * ((size_t)rp.stages * rp.stage_bytes + kSmemTail);
  const int threads = rp.subs * kThreads;
  static bool attr_done[64][2] = {};
  const int ti = std::is_same<T, __half>::value ? 1 : 0;
  if (!attr_done[h->device & 63][ti]) {
    DD_CUDA(h, cudaFuncSetAttribute(rollout_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024));
    attr_done[h->device & 63][ti] = true;
  }
  int per_sm = 0;
  // The occupancy calculator counts any kernel that allocates TMEM as one
  // CTA per SM, and a cooperative launch is held to that count.
  DD_CUDA(h, cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, rollout_kernel<T>, threads, smem));
  if (per_sm < 1) return DD_EUNSUPPORTED;
  const int grid = h->num_sms;
  if (grid * rp.subs > h->max_ctas) return DD_EUNSUPPORTED;
  RollMaps maps;
  maps.a[0] = h->tm_ws;
  maps.a[1] = h->tm_whh;
  maps.a[2] = h->tm_fc2;
  maps.b[0] = h->tm_h[0];
  maps.b[1] = h->tm_h[1];
  maps.b[2] = h->tm_mid;
  DD_CUDA(h, cudaMemsetAsync(h->rbar, 0, (size_t)(kMaxRollPhases + 1) * 4, st));
  int rc = timing_begin(h, DD_PHASE_ROLLOUT, st);
  if (rc) return rc;
  cudaLaunchConfig_t cfg{};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident: the phases wait on one another
  attr[0].val.cooperative = 1;
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  DD_CUDA(h, cudaLaunchKernelEx(&cfg, rollout_kernel<T>, maps, rp));
  return timing_end(h, st);
}

// The library links its own (static) CUDA runtime, whose current device is
// private to it: every entry point selects the handle's device itself.
int use_device(dd_handle* h) {
  DD_CUDA(h, cudaSetDevice(h->device));
  return DD_OK;
}

int check_ready(dd_handle* h) {
  if (!h) return DD_EINVAL;
  if (!h->have_weights) return fail(h, DD_EINVAL, "dd_set_weights has not been called");
  if (!h->w.table) return fail(h, DD_EINVAL, "weights.table is null (build it with dd_build_table)");
  return use_device(h);
}

void free_packed(dd_handle* h) {
  void** bufs[] = {&h->pk_wz, &h->pk_ws, &h->pk_fc2, &h->pk_whh, &h->pk_lm};
  for (void** b : bufs) {
    if (*b) cudaFree(*b);
    *b = nullptr;
  }
}

// Packed copy of W [rows x K] (row stride ld) for 1-D bulk streaming.
int pack_matrix(dd_handle* h, const void* w, long long rows, long long K, long long ld, void** out) {
  const int KC = ceil_div(K, kChunkK);
  const long long blocks = (long long)ceil_div(rows, kTileM) * KC;
  DD_CUDA(h, cudaMalloc(out, (size_t)blocks * kATileBytes));
  pack_tiles_kernel<<<(unsigned)blocks, 256>>>(static_cast<const uint16_t*>(w), rows, K, ld, KC,
                                               static_cast<uint4*>(*out));
  DD_CUDA(h, cudaGetLastError());
  return DD_OK;
}

// Launch-shape knobs from the environment (DD_RING_KB_*, DD_MIN_SMEM_KB_BIG,
// DD_CTAS_PER_SM_*, DD_PACK_WEIGHTS, DD_ROLLOUT_PERSISTENT,
// DD_MIN_UNITS_PER_CTA, DD_NACC, DD_TMEM_COLS, DD_L2_PREFETCH_KB, DD_FUSE_CELL, DD_BASE_STAGE,
// DD_WIDE_TWO_PER_SM, DD_WIDE_EPI_WARPS, DD_WIDE_PAIR, DD_L2_KEEP_MB, DD_EVEN_CUT_PCT, DD_BASE_BUFS, DD_WIDE_ONE_SLOT) over the defaults of a fresh
// handle.  dd_create and dd_rollout_noalloc both read them here, so the two
// entry points always build the same launches.
void read_launch_env(dd_handle* h) {
  auto env_int = [](const char* name, int def, int lo, int hi) {
    const char* v = getenv(name);
    if (!v || !*v) return def;
    const int x = atoi(v);
    return x < lo ? lo : (x > hi ? hi : x);
  };
  const dd_handle d{};
  h->ring_kb_big = env_int("DD_RING_KB_BIG", d.ring_kb_big, 36, 220);
  h->ring_kb_small = env_int("DD_RING_KB_SMALL", d.ring_kb_small, 36, 220);
  h->min_smem_kb_big = env_int("DD_MIN_SMEM_KB_BIG", d.min_smem_kb_big, 0, 227);
  h->ctas_per_sm_big = env_int("DD_CTAS_PER_SM_BIG", d.ctas_per_sm_big, 1, 2);
  h->ctas_per_sm_small = env_int("DD_CTAS_PER_SM_SMALL", d.ctas_per_sm_small, 1, 2);
  h->pack = env_int("DD_PACK_WEIGHTS", 0, 0, 1) != 0;
  h->rollout_mode = env_int("DD_ROLLOUT_PERSISTENT", 0, 0, 1) ? 0 : 1;
  h->min_units_per_cta = env_int("DD_MIN_UNITS_PER_CTA", d.min_units_per_cta, 1, 64);
  h->max_nacc = env_int("DD_NACC", d.max_nacc, 1, 4);
  h->tmem_cols_per_cta = env_int("DD_TMEM_COLS", d.tmem_cols_per_cta, 32, 512);
  h->l2_prefetch_kb = env_int("DD_L2_PREFETCH_KB", d.l2_prefetch_kb, 0, 4096);
  h->l2_keep_mb = env_int("DD_L2_KEEP_MB", d.l2_keep_mb, 0, 120);
  h->fuse_cell = env_int("DD_FUSE_CELL", d.fuse_cell, 0, 1);
  h->base_stage = env_int("DD_BASE_STAGE", d.base_stage, 0, 1);
  h->wide_two_per_sm = env_int("DD_WIDE_TWO_PER_SM", d.wide_two_per_sm, 0, 1);
  h->wide_epi_warps = env_int("DD_WIDE_EPI_WARPS", d.wide_epi_warps, 4, 8) == 8 ? 8 : 4;
  h->wide_pair = env_int("DD_WIDE_PAIR", d.wide_pair, 0, 1);
  h->even_cut_pct = env_int("DD_EVEN_CUT_PCT", d.even_cut_pct, 0, 101);
  h->base_bufs = env_int("DD_BASE_BUFS", d.base_bufs, 0, 2);
  h->wide_one_slot = env_int("DD_WIDE_ONE_SLOT", d.wide_one_slot, 0, 1);
}

}  // namespace

// ============================================================================ C ABI

// One verify launch.  The vocab of a row is cut into `parts` chunks so that
// the grid (parts x rows) is at most one wave of resident CTAs, with at least
// one group of vectors per thread in a chunk; chunks start on whole vectors.
template <typename T>
static int launch_verify(dd_handle* h, const T* logits, int dt, int32_t k1, const int64_t* verify_ids,
                         int64_t* posterior_out, int32_t* accept_out, int64_t* bonus_out, void* stream) {
  const dd_config& c = h->cfg;
  const long long rows = (long long)c.batch * k1;
  const cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (!h->verify_per_sm[dt]) {
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, verify_accept_kernel<T>, kVerifyThreads, 0) !=
            cudaSuccess ||
        per_sm < 1)
      return fail(h, DD_ECUDA, "verify_accept: occupancy query failed");
    h->verify_per_sm[dt] = per_sm;
  }
  constexpr int kVec = 16 / (int)sizeof(T);
  const long long slots = (long long)h->num_sms * h->verify_per_sm[dt];
  const int min_chunk = kVerifyThreads * kVerifyGroup * kVec;
  int parts = (int)std::max<long long>(1, slots / rows);
  parts = std::min(parts, std::max(1, c.vocab / min_chunk));
  const int chunk = ceil_div(ceil_div(c.vocab, parts), kVec) * kVec;
  Launch launch(dim3(ceil_div(c.vocab, chunk), (unsigned)rows), dim3(kVerifyThreads), 0, st);
  const cudaError_t e = cudaLaunchKernelEx(&launch.cfg, verify_accept_kernel<T>, logits, c.vocab, chunk, c.batch,
                                           (int)k1, verify_ids, posterior_out, accept_out, bonus_out, h->vwords,
                                           h->vdone, h->status);
  if (e != cudaSuccess) return fail(h, DD_ECUDA, "verify_accept launch: %s", cudaGetErrorString(e));
  return DD_OK;
}

extern "C" {

const char* dd_version(void) { return "domino_b200 0.1 (sm_100a, tcgen05 weight streaming)"; }

int dd_create(const dd_config* cfg, int device, dd_handle** out) {
  if (!cfg || !out) return fail(nullptr, DD_EINVAL, "null argument");
  *out = nullptr;
  const dd_config& c = *cfg;
  if (c.batch < 1 || c.batch > kMaxBatch)
    return fail(nullptr, DD_EINVAL, "batch %d outside [1, %d] (shard larger batches across handles)", c.batch,
                kMaxBatch);
  if (c.steps < 1 || c.hidden < 8 || c.gru_hidden < 8 || c.emb_dim < 8 || c.vocab < 2 || c.prefix_tokens < 1)
    return fail(nullptr, DD_EINVAL, "bad shape");
  if (c.hidden % 8 || c.gru_hidden % 8 || c.emb_dim % 8)
    return fail(nullptr, DD_EINVAL, "hidden, gru_hidden and emb_dim must be multiples of 8");
  if (c.dtype != DD_BF16 && c.dtype != DD_FP16 && c.dtype != DD_F32)
    return fail(nullptr, DD_EINVAL, "dtype must be DD_BF16, DD_FP16 or DD_F32");
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess)
    return fail(nullptr, DD_ECUDA, "cannot query device %d", device);
  if (prop.major != 10)
    return fail(nullptr, DD_EUNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a", device,
                prop.major, prop.minor);
  dd_handle* h = new dd_handle();
  h->device = device;
  h->cfg = c;
  h->es = c.dtype == DD_F32 ? 4 : 2;
  h->num_sms = prop.multiProcessorCount;
  h->N1 = round_up(c.batch, 16);
  h->N2 = round_up(2 * c.batch, 16);
  h->v_local = c.vocab;
  const int npre_max = c.prefix_tokens - 1;
  h->nslots = npre_max + c.steps;
  {
    // exchange buffer: argmax words, their flags, s / gh flags, then mid and gh
    const size_t words = (size_t)2 * h->nslots * kMaxRanks * c.batch;
    const size_t flags = (size_t)2 * h->nslots * kMaxRanks;
    h->xsflag_off = words + flags;  // u64 index
    size_t bytes = (words + 2 * flags) * 8;
    bytes = (bytes + 255) & ~size_t(255);
    h->xmid_off = bytes;
    bytes += ((size_t)h->N2 * c.emb_dim * 2 + 255) & ~size_t(255);
    h->xgh_off = bytes;  // (mid: N2 >= 2B rows of 2 bytes hold the fp32 [B, E] mid of fp32 heads too)
    bytes += ((size_t)c.batch * 3 * c.gru_hidden * h->es + 255) & ~size_t(255);
    h->xbuf_bytes = bytes;
  }
  h->max_tiles = ceil_div(c.vocab, kTileM) + ceil_div(c.emb_dim, kTileM) + ceil_div(3LL * c.gru_hidden, kTileM) + 1;
  read_launch_env(h);
  h->max_ctas = h->num_sms * std::max(h->ctas_per_sm_big, h->ctas_per_sm_small);
  int prev = 0;
  cudaGetDevice(&prev);
  auto cleanup_fail = [&](int code) {
    dd_destroy(h);
    cudaSetDevice(prev);
    return code;
  };
  if (cudaSetDevice(device) != cudaSuccess) return cleanup_fail(fail(nullptr, DD_ECUDA, "cudaSetDevice failed"));
  const size_t es = h->es;
  const size_t positions = (size_t)npre_max + c.steps;
  struct A {
    void** p;
    size_t bytes;
  } allocs[] = {
      {&h->zbuf, (size_t)c.batch * positions * c.emb_dim * es},
      {&h->hbuf[0], (size_t)h->N1 * c.gru_hidden * es},
      {&h->hbuf[1], (size_t)h->N1 * c.gru_hidden * es},
      {(void**)&h->slots, (size_t)c.batch * h->nslots * 8},
      {(void**)&h->partials, (size_t)2 * h->max_ctas * 256 * kTileM * 4},
      {(void**)&h->counters, (size_t)h->max_tiles * 4},
      {(void**)&h->status, 64},
      {(void**)&h->xbuf, h->xbuf_bytes},
      {(void**)&h->xsdone, (size_t)h->nslots * 4},
      {(void**)&h->xseq, 64},
      {(void**)&h->xdone, (size_t)h->nslots * 4},
      {(void**)&h->vwords, (size_t)c.batch * dd_handle::kMaxVerifyPositions * 8},
      {(void**)&h->vdone, 64},
      {(void**)&h->rbar, (size_t)(kMaxRollPhases + 1) * 4},
      {(void**)&h->gbar, 64},
  };
  for (auto& a : allocs) {
    if (cudaMalloc(a.p, a.bytes) != cudaSuccess)
      return cleanup_fail(fail(nullptr, DD_ECUDA, "cudaMalloc(%zu) failed", a.bytes));
    if (cudaMemset(*a.p, 0, a.bytes) != cudaSuccess)
      return cleanup_fail(fail(nullptr, DD_ECUDA, "cudaMemset failed"));
  }
  h->midbuf = reinterpret_cast<uint8_t*>(h->xbuf) + h->xmid_off;
  h->ghbuf = reinterpret_cast<uint8_t*>(h->xbuf) + h->xgh_off;
  int rc = DD_OK;
  if (c.dtype != DD_F32) {  // fp32 heads read their operands with plain loads
    rc = encode_kmajor(h, &h->tm_mid, h->midbuf, c.dtype, c.emb_dim, h->N2, c.emb_dim, h->N2);
    if (!rc) rc = encode_kmajor(h, &h->tm_h[0], h->hbuf[0], c.dtype, c.gru_hidden, h->N1, c.gru_hidden, h->N1);
    if (!rc) rc = encode_kmajor(h, &h->tm_h[1], h->hbuf[1], c.dtype, c.gru_hidden, h->N1, c.gru_hidden, h->N1);
  }
  if (rc) {
    snprintf(g_global_error, sizeof(g_global_error), "%s", h->err);
    return cleanup_fail(rc);
  }
  cudaSetDevice(prev);
  *out = h;
  return DD_OK;
}

int dd_set_weights(dd_handle* h, const dd_weights* w) {
  if (!h || !w) return DD_EINVAL;
  const dd_config& c = h->cfg;
  if (!w->fc1 || !w->fc2 || !w->w_hh) return fail(h, DD_EINVAL, "fc1, fc2 and w_hh are required");
  if (w->fc1_ld < c.hidden + c.gru_hidden || w->fc2_ld < c.emb_dim || w->w_hh_ld < c.gru_hidden)
    return fail(h, DD_EINVAL, "leading dimension smaller than the row length");
  if (w->table) {
    if (w->table_ld < 3LL * c.gru_hidden || (w->table_ld % 8) != 0 || (reinterpret_cast<uintptr_t>(w->table) & 15))
      return fail(h, DD_EINVAL, "table must be [V, 3G], 16-byte aligned, row stride a multiple of 8 elements");
  }
  if (c.dtype == DD_F32) {
    // fp32 heads: float4 loads of every weight row
    const void* ptrs[] = {w->fc1, w->fc2, w->w_hh, w->table, w->lm_head};
    const long long lds[] = {w->fc1_ld, w->fc2_ld, w->w_hh_ld, w->table ? w->table_ld : 0,
                             w->lm_head ? w->lm_head_ld : 0};
    for (int i = 0; i < 5; ++i)
      if ((ptrs[i] && (reinterpret_cast<uintptr_t>(ptrs[i]) & 15)) || (lds[i] & 3))
        return fail(h, DD_EINVAL, "fp32 weights must be 16-byte aligned with row strides a multiple of 4");
    if (w->lm_head && w->lm_head_ld < c.hidden) return fail(h, DD_EINVAL, "lm_head_ld smaller than the row length");
    h->w = *w;
    h->have_weights = true;
    return DD_OK;
  }
  const char* esz = reinterpret_cast<const char*>(w->fc1);
  int rc = encode_kmajor(h, &h->tm_wz, w->fc1, c.dtype, c.hidden, c.emb_dim, w->fc1_ld, kTileM);
  if (!rc) rc = encode_kmajor(h, &h->tm_ws, esz + (size_t)c.hidden * 2, c.dtype, c.gru_hidden, c.emb_dim, w->fc1_ld, kTileM);
  if (!rc) rc = encode_kmajor(h, &h->tm_fc2, w->fc2, c.dtype, c.emb_dim, h->v_local, w->fc2_ld, kTileM);
  if (!rc) rc = encode_kmajor(h, &h->tm_whh, w->w_hh, c.dtype, c.gru_hidden, 3LL * c.gru_hidden, w->w_hh_ld, kTileM);
  if (!rc && w->lm_head)
    rc = encode_kmajor(h, &h->tm_lm, w->lm_head, c.dtype, c.hidden, h->v_local, w->lm_head_ld, kTileM);
  if (rc) return rc;
  free_packed(h);
  if (h->pack) {
    // The weights may still be being written on another stream of this
    // process: wait for the device, pack, and wait for the packing.
    DD_CUDA(h, cudaDeviceSynchronize());
    const long long G = c.gru_hidden;
    rc = pack_matrix(h, w->fc1, c.emb_dim, c.hidden, w->fc1_ld, &h->pk_wz);
    if (!rc) rc = pack_matrix(h, esz + (size_t)c.hidden * 2, c.emb_dim, G, w->fc1_ld, &h->pk_ws);
    if (!rc) rc = pack_matrix(h, w->fc2, h->v_local, c.emb_dim, w->fc2_ld, &h->pk_fc2);
    if (!rc) rc = pack_matrix(h, w->w_hh, 3 * G, G, w->w_hh_ld, &h->pk_whh);
    if (!rc && w->lm_head) rc = pack_matrix(h, w->lm_head, h->v_local, c.hidden, w->lm_head_ld, &h->pk_lm);
    if (!rc) DD_CUDA(h, cudaDeviceSynchronize());
    if (rc) {
      free_packed(h);
      return rc;
    }
  }
  h->w = *w;
  h->have_weights = true;
  return DD_OK;
}

int dd_set_rollout_mode(dd_handle* h, int mode) {
  if (!h || mode < 0 || mode > 1) return DD_EINVAL;
  h->rollout_mode = mode;
  return DD_OK;
}

int dd_set_middle(dd_handle* h, int middle) {
  if (!h) return DD_EINVAL;
  if (middle < MID_SILU || middle > MID_SILU_ROUNDED) return fail(h, DD_EINVAL, "unknown middle kind %d", middle);
  h->middle = middle;
  return DD_OK;
}

int dd_set_weight_layout(dd_handle* h, int packed) {
  if (!h) return DD_EINVAL;
  h->pack = packed != 0;
  h->have_weights = false;  // dd_set_weights must run again
  return DD_OK;
}

int dd_build_table(dd_handle* h, const void* embed, int64_t embed_ld, const void* w_ih, int64_t w_ih_ld,
                   const void* b_ih, void* table_out, void* stream) {
  if (!h) return DD_EINVAL;
  const dd_config& c = h->cfg;
  if (!embed || !w_ih || !table_out) return fail(h, DD_EINVAL, "null argument");
  if (reinterpret_cast<uintptr_t>(table_out) & 15) return fail(h, DD_EINVAL, "table_out is not 16-byte aligned");
  int rc = use_device(h);
  if (rc) return rc;
  CUtensorMap tm_wih, tm_emb;
  if (c.dtype == DD_F32) {
    if ((reinterpret_cast<uintptr_t>(embed) & 15) || (reinterpret_cast<uintptr_t>(w_ih) & 15) || (embed_ld & 3) ||
        (w_ih_ld & 3))
      return fail(h, DD_EINVAL, "fp32 embed / w_ih must be 16-byte aligned with row strides a multiple of 4");
  } else {
    rc = encode_kmajor(h, &tm_wih, w_ih, c.dtype, c.hidden, 3LL * c.gru_hidden, w_ih_ld, kTileM);
    if (!rc) rc = encode_kmajor(h, &tm_emb, embed, c.dtype, c.hidden, c.vocab, embed_ld, wide_pair_pass(h, 256) ? 128 : 256);
    if (rc) return rc;
  }
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  for (int n_off = 0; n_off < c.vocab; n_off += 256) {
    GemvParams p = base_params(h);
    p.nseg = 1;
    p.seg[0] = {3 * c.gru_hidden, 0, EPI_TABLE};
    p.K = c.hidden;
    p.N = 256;
    p.b_box_rows = wide_pair_pass(h, 256) ? 128 : 256;
    p.n_off = n_off;
    p.n_valid = std::min(256, c.vocab - n_off);
    p.table_out = table_out;
    p.table_ld = 3LL * c.gru_hidden;
    p.b_ih = b_ih;
    p.w32[0] = static_cast<const float*>(w_ih);
    p.w32_ld[0] = w_ih_ld;
    p.x32 = static_cast<const float*>(embed);
    p.x32_ld = embed_ld;
    if (c.dtype == DD_F32)
      rc = launch_gemv<float, PH_TABLE>(h, tm_wih, nullptr, tm_emb, p, PhaseClass::Big, false, st);
    else if (c.dtype == DD_FP16)
      rc = launch_gemv<__half, PH_TABLE>(h, tm_wih, nullptr, tm_emb, p, PhaseClass::Big, false, st);
    else
      rc = launch_gemv<__nv_bfloat16, PH_TABLE>(h, tm_wih, nullptr, tm_emb, p, PhaseClass::Big, false, st);
    if (rc) return rc;
  }
  return DD_OK;
}

int dd_rollout(dd_handle* h, const int64_t* prefix_ids, const void* parallel_hiddens, const void* base_logits,
               int64_t* out_tokens, void* stream) {
  int rc = check_ready(h);
  if (rc) return rc;
  if (!prefix_ids || !parallel_hiddens || !base_logits || !out_tokens) return fail(h, DD_EINVAL, "null argument");
  const dd_config& c = h->cfg;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  DD_CUDA(h, cudaMemsetAsync(h->slots, 0, (size_t)c.batch * h->nslots * 8, st));
  rc = begin_exchange(h, st);
  if (rc) return rc;
  // base_logits rows are full-vocab rows; a vocab shard reads its own columns.
  const long long ld = c.vocab, voff = h->v_off;
  if (c.dtype == DD_F32) {
    rc = run_z_phase<float>(h, parallel_hiddens, c.steps, 0, nullptr, st);
    if (!rc)
      rc = run_rollout<float>(h, prefix_ids, c.prefix_tokens, c.prefix_tokens, 0, c.steps, base_logits, ld, voff,
                              out_tokens, c.steps, 0, nullptr, st);
  } else if (c.dtype == DD_FP16) {
    rc = run_z_phase<__half>(h, parallel_hiddens, c.steps, 0, nullptr, st);
    if (!rc)
      rc = run_rollout_persistent<__half>(h, prefix_ids, c.prefix_tokens, c.prefix_tokens, 0, c.steps, base_logits,
                                          ld, voff, out_tokens, c.steps, 0, nullptr, st);
    if (rc == DD_EUNSUPPORTED)
      rc = run_rollout<__half>(h, prefix_ids, c.prefix_tokens, c.prefix_tokens, 0, c.steps, base_logits, ld, voff,
                               out_tokens, c.steps, 0, nullptr, st);
  } else {
    rc = run_z_phase<__nv_bfloat16>(h, parallel_hiddens, c.steps, 0, nullptr, st);
    if (!rc)
      rc = run_rollout_persistent<__nv_bfloat16>(h, prefix_ids, c.prefix_tokens, c.prefix_tokens, 0, c.steps,
                                                 base_logits, ld, voff, out_tokens, c.steps, 0, nullptr, st);
    if (rc == DD_EUNSUPPORTED)
      rc = run_rollout<__nv_bfloat16>(h, prefix_ids, c.prefix_tokens, c.prefix_tokens, 0, c.steps, base_logits, ld,
                                      voff, out_tokens, c.steps, 0, nullptr, st);
  }
  return rc;
}

int dd_draft_block(dd_handle* h, const int64_t* last_token, const void* parallel_hiddens, void* base_logits_out,
                   int64_t* verify_out, void* stream) {
  int rc = check_ready(h);
  if (rc) return rc;
  if (!h->w.lm_head) return fail(h, DD_EINVAL, "weights.lm_head is null");
  if (!last_token || !parallel_hiddens || !base_logits_out || !verify_out) return fail(h, DD_EINVAL, "null argument");
  const dd_config& c = h->cfg;
  const int npre = c.prefix_tokens - 1;
  const int positions = npre + c.steps;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  DD_CUDA(h, cudaMemsetAsync(h->slots, 0, (size_t)c.batch * h->nslots * 8, st));
  rc = begin_exchange(h, st);
  if (rc) return rc;
  const int ld = positions + 1;
  // base_logits_out holds this rank's vocab columns only: rows of v_local.
  const long long bld = h->v_local;
  if (c.dtype == DD_F32) {
    rc = run_z_phase<float>(h, parallel_hiddens, positions, npre, base_logits_out, st);
    if (!rc)
      rc = run_rollout<float>(h, last_token, 1, 1, npre, positions, base_logits_out, bld, 0, verify_out, ld,
                              1 + npre, verify_out, st);
  } else if (c.dtype == DD_FP16) {
    rc = run_z_phase<__half>(h, parallel_hiddens, positions, npre, base_logits_out, st);
    if (!rc)
      rc = run_rollout_persistent<__half>(h, last_token, 1, 1, npre, positions, base_logits_out, bld, 0, verify_out,
                                          ld, 1 + npre, verify_out, st);
    if (rc == DD_EUNSUPPORTED)
      rc = run_rollout<__half>(h, last_token, 1, 1, npre, positions, base_logits_out, bld, 0, verify_out, ld,
                               1 + npre, verify_out, st);
  } else {
    rc = run_z_phase<__nv_bfloat16>(h, parallel_hiddens, positions, npre, base_logits_out, st);
    if (!rc)
      rc = run_rollout_persistent<__nv_bfloat16>(h, last_token, 1, 1, npre, positions, base_logits_out, bld, 0,
                                                 verify_out, ld, 1 + npre, verify_out, st);
    if (rc == DD_EUNSUPPORTED)
      rc = run_rollout<__nv_bfloat16>(h, last_token, 1, 1, npre, positions, base_logits_out, bld, 0, verify_out,
                                      ld, 1 + npre, verify_out, st);
  }
  return rc;
}

int dd_accept(const int64_t* verify_ids, const int64_t* posterior, int32_t batch, int32_t k1, int32_t* accept_out,
              int64_t* bonus_out, void* stream) {
  if (!verify_ids || !posterior || !accept_out || !bonus_out || batch < 1 || k1 < 1)
    return fail(nullptr, DD_EINVAL, "bad accept arguments");
  cudaPointerAttributes attr;
  if (cudaPointerGetAttributes(&attr, verify_ids) != cudaSuccess || attr.type != cudaMemoryTypeDevice)
    return fail(nullptr, DD_EINVAL, "verify_ids is not device memory");
  if (cudaSetDevice(attr.device) != cudaSuccess) return fail(nullptr, DD_ECUDA, "cudaSetDevice failed");
  Launch L(dim3(ceil_div(batch, 128)), dim3(128), 0, reinterpret_cast<cudaStream_t>(stream));
  cudaError_t e = cudaLaunchKernelEx(&L.cfg, accept_kernel, verify_ids, posterior, (int)batch, (int)k1, accept_out,
                                     bonus_out);
  if (e != cudaSuccess) return fail(nullptr, DD_ECUDA, "accept launch: %s", cudaGetErrorString(e));
  return DD_OK;
}

int dd_verify_accept(dd_handle* h, const void* target_logits, int32_t logits_dtype, int32_t k1,
                     const int64_t* verify_ids, int64_t* posterior_out, int32_t* accept_out, int64_t* bonus_out,
                     void* stream) {
  if (!h) return DD_EINVAL;
  if (!target_logits || !verify_ids || !posterior_out || !accept_out || !bonus_out)
    return fail(h, DD_EINVAL, "dd_verify_accept: null argument");
  if (k1 < 1 || k1 > dd_handle::kMaxVerifyPositions)
    return fail(h, DD_EINVAL, "dd_verify_accept: %d positions outside [1, %d]", k1, dd_handle::kMaxVerifyPositions);
  int rc = use_device(h);
  if (rc) return rc;
  if (logits_dtype == DD_F32) return launch_verify<float>(h, static_cast<const float*>(target_logits), 0, k1,
                                                          verify_ids, posterior_out, accept_out, bonus_out, stream);
  if (logits_dtype == DD_FP16) return launch_verify<__half>(h, static_cast<const __half*>(target_logits), 1, k1,
                                                            verify_ids, posterior_out, accept_out, bonus_out, stream);
  if (logits_dtype == DD_BF16)
    return launch_verify<__nv_bfloat16>(h, static_cast<const __nv_bfloat16*>(target_logits), 2, k1, verify_ids,
                                        posterior_out, accept_out, bonus_out, stream);
  return fail(h, DD_EINVAL, "dd_verify_accept: logits dtype %d", logits_dtype);
}

int dd_get_exchange_buffer(dd_handle* h, void** dev_ptr, uint64_t* bytes) {
  if (!h || !dev_ptr) return DD_EINVAL;
  *dev_ptr = h->xbuf;
  if (bytes) *bytes = h->xbuf_bytes;
  return DD_OK;
}

int dd_ipc_export(const void* dev_ptr, void* handle_out) {
  if (!dev_ptr || !handle_out) return fail(nullptr, DD_EINVAL, "dd_ipc_export: null argument");
  cudaPointerAttributes attr;
  if (cudaPointerGetAttributes(&attr, dev_ptr) != cudaSuccess || attr.type != cudaMemoryTypeDevice)
    return fail(nullptr, DD_EINVAL, "dd_ipc_export: not device memory");
  if (cudaSetDevice(attr.device) != cudaSuccess) return fail(nullptr, DD_ECUDA, "cudaSetDevice failed");
  cudaIpcMemHandle_t ipc;
  const cudaError_t e = cudaIpcGetMemHandle(&ipc, const_cast<void*>(dev_ptr));
  if (e != cudaSuccess) return fail(nullptr, DD_ECUDA, "cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
  memcpy(handle_out, &ipc, sizeof(ipc));
  return DD_OK;
}

int dd_ipc_open(int device, const void* handle_in, void** dev_ptr_out) {
  if (!handle_in || !dev_ptr_out) return fail(nullptr, DD_EINVAL, "dd_ipc_open: null argument");
  if (cudaSetDevice(device) != cudaSuccess) return fail(nullptr, DD_ECUDA, "cudaSetDevice failed");
  cudaIpcMemHandle_t ipc;
  memcpy(&ipc, handle_in, sizeof(ipc));
  const cudaError_t e = cudaIpcOpenMemHandle(dev_ptr_out, ipc, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return fail(nullptr, DD_ECUDA, "cudaIpcOpenMemHandle: %s", cudaGetErrorString(e));
  return DD_OK;
}

int dd_ipc_close(int device, void* dev_ptr) {
  if (!dev_ptr) return DD_OK;
  if (cudaSetDevice(device) != cudaSuccess) return fail(nullptr, DD_ECUDA, "cudaSetDevice failed");
  const cudaError_t e = cudaIpcCloseMemHandle(dev_ptr);
  if (e != cudaSuccess) return fail(nullptr, DD_ECUDA, "cudaIpcCloseMemHandle: %s", cudaGetErrorString(e));
  return DD_OK;
}

int dd_set_vocab_shard(dd_handle* h, int32_t rank, int32_t world, int64_t vocab_begin, int64_t vocab_end,
                       void* const* peer_exchange_buffers) {
  if (!h) return DD_EINVAL;
  if (world < 1 || world > kMaxRanks || rank < 0 || rank >= world)
    return fail(h, DD_EINVAL, "rank %d / world %d outside [0, %d)", rank, world, kMaxRanks);
  if (vocab_begin < 0 || vocab_end <= vocab_begin || vocab_end > h->cfg.vocab)
    return fail(h, DD_EINVAL, "vocab shard [%lld, %lld) outside [0, %d)", (long long)vocab_begin,
                (long long)vocab_end, h->cfg.vocab);
  if (world > 1 && !peer_exchange_buffers) return fail(h, DD_EINVAL, "peer exchange buffers are required");
  if (world > 1 && h->cfg.dtype == DD_F32) return fail(h, DD_EUNSUPPORTED, "vocab sharding needs bf16 / fp16 weights");
  for (int j = 0; j < kMaxRanks; ++j) h->peer[j] = nullptr;
  for (int j = 0; j < world; ++j) {
    void* pj = (world == 1 || j == rank) ? h->xbuf : peer_exchange_buffers[j];
    if (!pj) return fail(h, DD_EINVAL, "exchange buffer of rank %d is null", j);
    h->peer[j] = static_cast<unsigned long long*>(pj);
  }
  h->world = world;
  h->rank = rank;
  h->v_off = (int)vocab_begin;
  h->v_local = (int)(vocab_end - vocab_begin);
  // s / gh slices: contiguous near-equal runs of 128-row tiles
  const int te = ceil_div(h->cfg.emb_dim, kTileM), tg = ceil_div(3LL * h->cfg.gru_hidden, kTileM);
  h->sgh_sharded = world > 1 && te >= world && tg >= world;
  for (int j = 0; j < world; ++j) {
    auto split = [&](int tiles, int rows, int* lo, int* hi) {
      const int base = tiles / world, extra = tiles % world;
      const int t0 = j * base + std::min(j, extra), t1 = t0 + base + (j < extra ? 1 : 0);
      *lo = std::min(rows, t0 * kTileM);
      *hi = std::min(rows, t1 * kTileM);
    };
    split(te, h->cfg.emb_dim, &h->e0[j], &h->e1[j]);
    split(tg, 3 * h->cfg.gru_hidden, &h->g0[j], &h->g1[j]);
  }
  h->have_weights = false;  // fc2 / lm_head must be given again as this rank's rows
  return DD_OK;
}

int dd_set_exchange_timeout(dd_handle* h, uint64_t timeout_ns) {
  if (!h || timeout_ns == 0) return DD_EINVAL;
  h->xtimeout_ns = timeout_ns;
  return DD_OK;
}

int dd_set_trace(dd_handle* h, const dd_trace* t) {
  if (!h) return DD_EINVAL;
  if (t && h->world > 1) return fail(h, DD_EINVAL, "dd_set_trace: vocab-sharded handles hold only slices of s and gh");
  h->tracing = t != nullptr;
  h->trace = t ? *t : dd_trace{};
  return DD_OK;
}

int dd_set_timing(dd_handle* h, int enable) {
  if (!h) return DD_EINVAL;
  h->timing = enable != 0;
  h->n_timed = 0;
  return DD_OK;
}

int dd_read_timing(dd_handle* h, int32_t* kinds, float* ms, int32_t max_records) {
  if (!h || (max_records > 0 && (!kinds || !ms))) return DD_EINVAL;
  int rc = use_device(h);
  if (rc) return rc;
  const int n = std::min<int>(h->n_timed, max_records);
  for (int i = 0; i < n; ++i) {
    DD_CUDA(h, cudaEventSynchronize(h->ev[2 * i + 1]));
    float t = 0.0f;
    DD_CUDA(h, cudaEventElapsedTime(&t, h->ev[2 * i], h->ev[2 * i + 1]));
    kinds[i] = h->timed_kind[i];
    ms[i] = t;
  }
  h->n_timed = 0;
  return n;
}

int dd_get_status(dd_handle* h) {
  if (!h) return DD_EINVAL;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(h->device);
  unsigned int s = 0;
  cudaError_t e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemcpy(&s, h->status, 4, cudaMemcpyDeviceToHost);
  if (e == cudaSuccess) e = cudaMemset(h->status, 0, 4);
  cudaSetDevice(prev);
  if (e != cudaSuccess) return fail(h, DD_ECUDA, "dd_get_status: %s", cudaGetErrorString(e));
  return (int)s;
}

const char* dd_last_error(const dd_handle* h) { return h ? h->err : g_global_error; }

int dd_destroy(dd_handle* h) {
  if (!h) return DD_OK;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(h->device);
  // (midbuf and ghbuf live inside xbuf)
  void* ptrs[] = {h->zbuf, h->hbuf[0], h->hbuf[1], h->slots, h->partials, h->counters, h->status, h->xbuf,
                  h->xseq, h->xdone,   h->xsdone,   h->vwords, h->vdone,    h->rbar,     h->gbar};
  for (void* p : ptrs)
    if (p) cudaFree(p);
  free_packed(h);
  for (cudaEvent_t e : h->ev)
    if (e) cudaEventDestroy(e);
  cudaSetDevice(prev);
  delete h;
  return DD_OK;
}

}  // extern "C"

// ============================================================================ allocation-free rollout
//
// dd_rollout_noalloc: the rollout of dd_rollout for callers that cannot
// allocate device memory -- code that runs while a CUDA graph is being
// captured (cudaMalloc is not allowed there), a host that has handed all of
// HBM to its own memory pool and treats any other allocation as a leak, or
// a stateless foreign-function binding that has no place to keep a handle
// and its buffers alive between calls.  Its scratch lives in the file-scope
// array below instead of in cudaMalloc'd handle buffers.

namespace {
constexpr size_t kNoAllocScratchBytes = size_t(32) << 20;  // 32 MiB
constexpr int kNoAllocMaxDevices = 16;
constexpr size_t kNoAllocStatusBytes = 256;  // the status word, at offset 0
}  // namespace

// One copy per device that loads this library's kernels, held until exit.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

namespace {

struct NoAllocDevice {
  bool ready = false;
  unsigned char* base = nullptr;  // device address of g_noalloc_scratch on this device
  int num_sms = 0;
  dd_handle h;                    // launch state pointing into g_noalloc_scratch
};
NoAllocDevice g_noalloc[kNoAllocMaxDevices];
std::mutex g_noalloc_mu;

int noalloc_fail(dd_handle* h, int rc) {
  if (h && h->err[0]) snprintf(g_global_error, sizeof(g_global_error), "%s", h->err);
  return rc;
}

}  // namespace

extern "C" int dd_rollout_noalloc(const dd_config* cfg, const dd_weights* w, int device, const int64_t* prefix_ids,
                                  const void* parallel_hiddens, const void* base_logits, int64_t* out_tokens,
                                  void* stream) {
  if (!cfg || !w || !prefix_ids || !parallel_hiddens || !base_logits || !out_tokens)
    return fail(nullptr, DD_EINVAL, "dd_rollout_noalloc: null argument");
  if (device < 0 || device >= kNoAllocMaxDevices)
    return fail(nullptr, DD_EINVAL, "dd_rollout_noalloc: device %d outside [0, %d)", device, kNoAllocMaxDevices);
  const dd_config& c = *cfg;
  if (c.batch < 1 || c.batch > kMaxBatch || c.steps < 1 || c.hidden < 8 || c.gru_hidden < 8 || c.emb_dim < 8 ||
      c.vocab < 2 || c.prefix_tokens < 1 || c.hidden % 8 || c.gru_hidden % 8 || c.emb_dim % 8 ||
      (c.dtype != DD_BF16 && c.dtype != DD_FP16 && c.dtype != DD_F32))
    return fail(nullptr, DD_EINVAL, "dd_rollout_noalloc: bad config (same rules as dd_create)");

  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  NoAllocDevice& d = g_noalloc[device];
  if (cudaSetDevice(device) != cudaSuccess) return fail(nullptr, DD_ECUDA, "dd_rollout_noalloc: cudaSetDevice failed");
  if (!d.ready) {
    // Once per device, with that device current: the device address of the
    // static scratch.  (The host-side symbol is only a stand-in and must
    // never be passed to a kernel.)
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, device) != cudaSuccess)
      return fail(nullptr, DD_ECUDA, "dd_rollout_noalloc: cannot query device %d", device);
    if (prop.major != 10)
      return fail(nullptr, DD_EUNSUPPORTED, "dd_rollout_noalloc: device %d is sm_%d%d, not sm_100", device,
                  prop.major, prop.minor);
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return fail(nullptr, DD_ECUDA, "dd_rollout_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    d.base = static_cast<unsigned char*>(p);
    d.num_sms = prop.multiProcessorCount;
    d.ready = true;
  }

  // Launch state for this call, laid out like dd_create's buffers.
  dd_handle& h = d.h;
  h.device = device;
  h.num_sms = d.num_sms;
  h.cfg = c;
  h.have_weights = false;
  h.timing = false;
  h.tracing = false;
  h.n_timed = 0;
  h.err[0] = 0;
  h.N1 = round_up(c.batch, 16);
  h.N2 = round_up(2 * c.batch, 16);
  h.es = c.dtype == DD_F32 ? 4 : 2;
  h.v_off = 0;
  h.v_local = c.vocab;  // unsharded
  h.world = 1;
  h.rank = 0;
  const int npre_max = c.prefix_tokens - 1;
  h.nslots = npre_max + c.steps;
  h.max_tiles = ceil_div(c.vocab, kTileM) + ceil_div(c.emb_dim, kTileM) + ceil_div(3LL * c.gru_hidden, kTileM) + 1;
  read_launch_env(&h);
  h.pack = false;      // packing would allocate: stream the caller's row-major weights
  h.rollout_mode = 1;  // one launch per phase: the persistent kernel's grid counters are not in this scratch
  h.max_ctas = h.num_sms * std::max(h.ctas_per_sm_big, h.ctas_per_sm_small);
  // Widest accumulator any split tile of a rollout can have.
  const int n_part = std::max(std::min(256, round_up(c.batch * c.steps, 16)), std::max(h.N1, h.N2));
  const size_t positions = (size_t)npre_max + c.steps;
  // The status word sits at a fixed place, the first 256 bytes, so that
  // dd_noalloc_status can find it whatever the shapes of the last call.
  size_t off = kNoAllocStatusBytes;
  auto take = [&](size_t bytes) {
    unsigned char* p = d.base + off;
    off = (off + bytes + 255) & ~size_t(255);
    return p;
  };
  h.status = reinterpret_cast<unsigned int*>(d.base);
  const size_t es = h.es;
  h.zbuf = take((size_t)c.batch * positions * c.emb_dim * es);
  h.midbuf = take((size_t)h.N2 * c.emb_dim * 2);  // N2 >= 2B rows: also holds fp32 [B, E]
  h.hbuf[0] = take((size_t)h.N1 * c.gru_hidden * es);
  h.hbuf[1] = take((size_t)h.N1 * c.gru_hidden * es);
  h.ghbuf = take((size_t)c.batch * 3 * c.gru_hidden * es);
  h.slots = reinterpret_cast<unsigned long long*>(take((size_t)c.batch * h.nslots * 8));
  h.partials = reinterpret_cast<float*>(take((size_t)2 * h.max_ctas * n_part * kTileM * 4));
  h.counters = reinterpret_cast<unsigned int*>(take((size_t)h.max_tiles * 4));
  h.gbar = reinterpret_cast<unsigned int*>(take(64));
  if (off > kNoAllocScratchBytes)
    return fail(nullptr, DD_EINVAL,
                "dd_rollout_noalloc: these shapes need %zu bytes of scratch; the static scratch holds %zu "
                "(use dd_create/dd_rollout instead)",
                off, kNoAllocScratchBytes);

  // The scratch keeps the previous call's contents: clear what must start at
  // zero (operand padding rows, split-tile counters).  The status word is
  // left alone: it collects the bits of every call until dd_noalloc_status
  // reads and clears it.
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const struct {
    void* p;
    size_t n;
  } zero[] = {{h.midbuf, (size_t)h.N2 * c.emb_dim * 2},
              {h.hbuf[0], (size_t)h.N1 * c.gru_hidden * es},
              {h.hbuf[1], (size_t)h.N1 * c.gru_hidden * es},
              {h.counters, (size_t)h.max_tiles * 4},
              {h.gbar, 64}};
  for (const auto& z : zero)
    if (cudaMemsetAsync(z.p, 0, z.n, st) != cudaSuccess)
      return fail(nullptr, DD_ECUDA, "dd_rollout_noalloc: cudaMemsetAsync failed");

  int rc = DD_OK;
  if (c.dtype != DD_F32) {
    rc = encode_kmajor(&h, &h.tm_mid, h.midbuf, c.dtype, c.emb_dim, h.N2, c.emb_dim, h.N2);
    if (!rc) rc = encode_kmajor(&h, &h.tm_h[0], h.hbuf[0], c.dtype, c.gru_hidden, h.N1, c.gru_hidden, h.N1);
    if (!rc) rc = encode_kmajor(&h, &h.tm_h[1], h.hbuf[1], c.dtype, c.gru_hidden, h.N1, c.gru_hidden, h.N1);
  }
  if (!rc) rc = dd_set_weights(&h, w);
  if (!rc) rc = dd_rollout(&h, prefix_ids, parallel_hiddens, base_logits, out_tokens, stream);
  return rc ? noalloc_fail(&h, rc) : DD_OK;
}

extern "C" int dd_noalloc_status(int device) {
  if (device < 0 || device >= kNoAllocMaxDevices)
    return fail(nullptr, DD_EINVAL, "dd_noalloc_status: device %d outside [0, %d)", device, kNoAllocMaxDevices);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  const NoAllocDevice& d = g_noalloc[device];
  if (!d.ready) return 0;  // no allocation-free call has run on this device
  int prev = 0;
  cudaGetDevice(&prev);
  if (cudaSetDevice(device) != cudaSuccess) return fail(nullptr, DD_ECUDA, "dd_noalloc_status: cudaSetDevice failed");
  unsigned int s = 0;
  cudaError_t e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemcpy(&s, d.base, sizeof(s), cudaMemcpyDeviceToHost);
  if (e == cudaSuccess) e = cudaMemset(d.base, 0, sizeof(s));
  cudaSetDevice(prev);
  if (e != cudaSuccess) return fail(nullptr, DD_ECUDA, "dd_noalloc_status: %s", cudaGetErrorString(e));
  return (int)s;
}
