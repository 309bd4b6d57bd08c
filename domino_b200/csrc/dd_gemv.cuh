// dd_gemv.cuh -- the weight-streaming tcgen05 kernel behind every contraction
// of the draft step.
//
// Shape of the problem.  Each phase of the draft step multiplies one or two
// weight matrices W [R x K] (bf16/fp16, row-major, K contiguous) by a small
// activation matrix X [N x K] (N = batch rows, or batch x positions) and
// hands the R x N result to an epilogue.  The weights are read exactly once
// per phase and dominate the bytes (the draft step is HBM-bound up to
// batch 32), so the kernel is built around keeping HBM busy:
//
//   * two CTAs per SM (persistent; measured faster than one CTA with a
//     deeper ring), 192 threads each:
//       warp 0      TMA producer: 128x64 weight tiles (16 KB, 128B-swizzled,
//                   L2 evict_first) + the matching 64-wide slice of X
//                   (N x 128 B, L2 evict_last: every CTA reuses it);
//       warp 1      TMEM allocator and the single MMA-issuing thread:
//                   tcgen05.mma kind::f16, M = 128 weight rows, N = X rows,
//                   K = 16 per instruction, fp32 accumulators in TMEM;
//       warps 2..5  epilogue: tcgen05.ld the 128 x N accumulator (one weight
//                   row per thread) and apply the phase's epilogue.
//   * stream-K partition: the phase's (tile, 64-wide k-chunk) units are cut
//     into gridDim.x equal contiguous ranges, so every SM streams the same
//     number of bytes (the vocab 151936 = 128 x 1187 does not divide into
//     148 tiles evenly; splitting along K does).  A tile whose units span
//     several CTAs is finished by the last of them to arrive: each writes its
//     fp32 partial to scratch, and the last sums all partials in CTA order,
//     so the result does not depend on arrival order.
//   * programmatic dependent launch: weights never depend on the previous
//     kernel, so the producer issues the first ring's worth of weight loads
//     before griddepcontrol.wait and only the activation loads after it; the
//     kernel also triggers its dependents at once, so the next phase's CTAs
//     sit beside this one and prefetch their own weights while this phase
//     drains.
//
// Every wait is bounded (kWaitLimitNs); a timeout sets DD_STATUS_TIMEOUT,
// unwinds all roles, drains in-flight TMA/MMA and frees TMEM.
#pragma once

#include "dd_cell_core.cuh"

namespace dd {

enum EpiKind : int {
  EPI_LMHEAD = 1,      // base[n, v] = acc (rounded); optional prefix argmax
  EPI_ZPROJ = 2,       // z[n, e] = acc + fc1_bias[e] (rounded)
  EPI_SPROJ_MID = 3,   // s = acc (rounded); mid = SiLU(z_t + s) -> (hi, lo) rows 2b, 2b+1
  EPI_GH = 4,          // gh[b, j] = acc + b_hh[j] (rounded)
  EPI_FC2_ARGMAX = 5,  // logit = acc(hi) + acc(lo) + fc2_bias + base_t -> atomicMax key
  EPI_TABLE = 6,       // table[n, j] = acc + b_ih[j] (rounded)
};

constexpr int kThreads = 192;
constexpr int kEpiWarp0 = 2;
constexpr int kTileM = 128;
constexpr int kChunkK = 64;
constexpr uint32_t kATileBytes = kTileM * 128;  // 16 KB
constexpr int kMaxStages = 16;
constexpr int kMaxBatch = 32;
constexpr uint32_t kSmemTail = 2048;            // barriers + flags + argmax reduction
// Staging area after the tail in phases whose epilogue writes X-row-major
// outputs (z, base logits, the W_ih table): one 16-column chunk of a tile,
// 16 x 128 elements of at most 4 bytes.
constexpr uint32_t kXposeBytes = 16 * 128 * 4;

struct GemvSeg {
  int rows;     // rows of W this phase streams
  int tiles;
  int kind;
  int row_off;  // W row (and output index) of the segment's first row; a multiple of 128
};

struct GemvParams {
  GemvSeg seg[2];
  // Packed weights (see pack_tiles_kernel): segment s's (tile, k-chunk) block
  // is the 16 KB at packed[s] + (tile * KC + kc) * 16384, already in the
  // swizzled order the MMA reads; null = load the row-major matrix by TMA.
  const uint8_t* packed[2];
  int nseg;
  int K, KC;
  int N;             // MMA N: X rows per pass, multiple of 16, <= 256
  int n_off;         // first X row of this pass
  int n_valid;       // X rows of this pass that carry data (<= N)
  long long units;   // (tile, k-chunk) units in this pass; CTA pairs: (256-row pair tile, k-chunk)
  long long tiles128;  // CTA pairs: the 128-row tiles of all segments (a pair tile past them is empty)
  int b_box_rows;    // rows of tmB's box: N, or N / 2 when the caller encoded it for CTA pairs
  int stages;
  // PH_FC2 with more than four batch rows: the producer also loads each tile's
  // base logits [B, 128] by TMA (the tensor map in tmA1) into one of two
  // buffers of base_stage_bytes after the tail; 0 = plain loads in the epilogue
  uint32_t base_stage_bytes;
  int base_bufs;     // 1 or 2 base-logit buffers (one frees the room of a fourth ring stage at batch 32)
  int l2_prefetch_units;  // weight tiles past the ring this CTA prefetches into L2 before waiting on its predecessor
  int w_keep[2];     // segment s's weights are loaded with L2 evict_last (kept for the next step) instead of evict_first
  uint32_t stage_bytes;
  uint32_t b_bytes;
  int acc_slots;
  uint32_t xpose_bytes;  // > 0: a kXposeBytes staging area follows the tail
  int nacc;          // independent accumulators per slot; K-step i goes to accumulator i % nacc
  uint32_t tmem_cols;
  uint32_t idesc;
  int B, t, V, E, G3;
  // EPI_LMHEAD: base_out[(n_off+n) * V + v]; prefix argmax where (n_off+n) % kpos < npre
  void* base_out;
  int kpos, npre;
  unsigned long long* slots;  // [B, nslots]: prefix i < npre, rollout step npre + t
  int nslots;
  // EPI_ZPROJ
  void* z_out;
  const void* fc1_bias;
  // EPI_SPROJ_MID: z_src[(b * z_rows_per_b + z_pos_off + t) * E + e]
  const void* z_src;
  int z_rows_per_b, z_pos_off;
  void* mid_out;
  void* s_out;  // optional trace: s[b * E + e] (rounded), as the epilogue uses it
  int middle;   // MID_*: the activation between fc1 and fc2, and with it the numerics (dd_ptx.cuh)
  // EPI_GH
  void* gh_out;
  const void* b_hh;
  // EPI_FC2_ARGMAX: base_src[(b * base_rows_per_b + base_pos_off + t) * V + v]
  const void* base_src;
  int base_rows_per_b, base_pos_off;
  const void* fc2_bias;
  // EPI_TABLE
  void* table_out;
  long long table_ld;
  const void* b_ih;
  // stream-K scratch, status
  float* partials;
  unsigned int* tile_counters;
  unsigned int* status;
  // vocab sharding: this rank's rows are global vocab ids v_off + row; base
  // logits rows have stride base_ld (input) / base_out_ld (output) and this
  // rank's slice starts at column base_voff of an input row.
  int v_off;
  long long base_ld, base_out_ld, base_voff;
  Exchange xchg;
  // PH_FC2: run the step's GRU cell in this launch, after a grid-wide
  // barrier (gbar: [0] arrival count, [1] generation) instead of in a launch
  // of its own
  int fused_cell;
  unsigned int* gbar;
  CellParams cell;
  int xslot0, xslot1;  // argmax words this launch publishes to every rank
  int sflag_slot;      // >= 0: this s / gh launch raises its step flag on every rank when done
  // fp32 heads (gemv_f32_kernel): the segments' weights and the X rows as
  // plain pointers, row strides in elements.
  const float* w32[2];
  long long w32_ld[2];
  const float* x32;
  long long x32_ld;
};

// CTA c's units are [unit_begin(c), unit_begin(c + 1)): equal contiguous
// ranges when there are at least as many units as CTAs; otherwise one unit
// each for the first U CTAs, so that CTAs without work only come last.
__device__ __forceinline__ long long unit_begin(int c, long long U, int G) {
  return U >= G ? (long long)c * U / G : (c < U ? c : U);
}

__device__ __forceinline__ int cta_of_unit(long long u, long long U, int G) {
  if (U < G) return (int)u;
  int c = (int)((u * G) / U);
  if (c >= G) c = G - 1;
  while (c + 1 < G && unit_begin(c + 1, U, G) <= u) ++c;
  while (c > 0 && unit_begin(c, U, G) > u) --c;
  return c;
}

// Scratch slot of CTA c's partial for tile T: each CTA owns two slots, one
// for the tile its range starts in and one for the tile it ends in.
__device__ __forceinline__ int partial_slot(int c, long long T, long long U, int G, int KC) {
  return 2 * c + ((unit_begin(c, U, G) / KC == T) ? 0 : 1);
}

__device__ __forceinline__ bool named_bar_and(uint32_t id, uint32_t nthreads, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)pred), "r"(id), "r"(nthreads)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ unsigned long long warp_max_u64(unsigned long long k) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    unsigned long long other = __shfl_xor_sync(0xFFFFFFFFu, k, o);
    k = other > k ? other : k;
  }
  return k;
}

__device__ __forceinline__ bool wait_ns(uint64_t* bar, uint32_t parity, uint64_t limit_ns) {
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > limit_ns) return false;
  }
  return true;
}

// One arrival of the calling CTA at a grid-wide barrier over n CTAs
// (bar[0] arrival count, bar[1] generation), then, if `wait`, a bounded wait
// for the last arrival.  The last CTA to arrive zeroes the count and bumps the
// generation, so the barrier resets itself and a launch replayed from a CUDA
// graph reuses it unchanged.  Every CTA of the grid must be resident at once
// (a one-wave grid whose dependents launch only after all of its CTAs have
// started).  Returns false if the wait gave up.
__device__ __forceinline__ bool grid_barrier(unsigned int* bar, unsigned int n, bool wait) {
  volatile unsigned int* gen = bar + 1;
  const unsigned int g0 = *gen;  // read before arriving: it cannot have moved yet
  __threadfence();
  if (atomicAdd(bar, 1u) == n - 1) {
    atomicExch(bar, 0u);
    __threadfence();
    atomicAdd(bar + 1, 1u);
    return true;
  }
  if (!wait) return true;
  const uint64_t t0 = globaltimer_ns();
  while (*gen == g0) {
    if (globaltimer_ns() - t0 > kWaitLimitNs) return false;
    __nanosleep(32);
  }
  __threadfence();
  return true;
}

// Context an epilogue thread needs to read its (possibly split) accumulator.
struct AccView {
  uint32_t taddr = 0;        // TMEM address of this thread's lane, column 0 of the slot
  int nacc = 1;              // accumulators of the slot, N columns apart
  bool combine = false;      // split tile finished here: sum partials of all segments
  int nseg = 1, myseg = 0, c_lo = 0;
  long long T = 0;
  const float* partials = nullptr;
  int N = 0;
  int r = 0;                 // row within the tile
  long long U = 0;
  int G = 0, KC = 0;
  uint32_t bar = 1;          // named barrier of the 128 epilogue threads
  void* xpose = nullptr;     // shared staging chunk for row-contiguous stores, or null
  long long row0 = 0;        // global row of the tile's first row
  long long row_end = 0;     // end of the segment's rows (exclusive, global)
  const void* bsm = nullptr; // PH_FC2 staging: this tile's base logits [B][128] in shared memory, or null
  int grp = 0, ngroups = 1;  // X-row-major outputs: this warpgroup takes 16-column chunks grp, grp + ngroups, ...
  int pmul = 1, padd = 0;    // partial scratch slot = partial_slot(...) * pmul + padd (CTA pairs: 2, rank)
};

// Four consecutive elements (8 or 16 bytes, aligned) from shared to global memory.
template <typename T>
__device__ __forceinline__ void store4(T* dst, const T* src) {
  if constexpr (sizeof(T) == 2)
    *reinterpret_cast<uint2*>(dst) = *reinterpret_cast<const uint2*>(src);
  else
    *reinterpret_cast<float4*>(dst) = *reinterpret_cast<const float4*>(src);
}

// This CTA's part of 16 accumulator columns [ch*16, ch*16+16): the sum of the
// slot's accumulators in a fixed order.
__device__ __forceinline__ void acc_local(const AccView& a, int ch, float* t) {
  tmem_ld16(a.taddr + ch * 16, *reinterpret_cast<float(*)[16]>(t));
  tmem_ld_wait();
  for (int i = 1; i < a.nacc; ++i) {
    float u[16];
    tmem_ld16(a.taddr + i * a.N + ch * 16, u);
    tmem_ld_wait();
#pragma unroll
    for (int j = 0; j < 16; ++j) t[j] += u[j];
  }
}

// 16 accumulator columns [ch*16, ch*16+16) of this thread's row, summed over
// the tile's segments in CTA order when the tile was split.
__device__ __forceinline__ void acc_chunk(const AccView& a, int ch, float* v) {
  float t[16];
  acc_local(a, ch, t);
  if (!a.combine) {
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = t[j];
    return;
  }
#pragma unroll
  for (int j = 0; j < 16; ++j) v[j] = 0.0f;
  for (int s = 0; s < a.nseg; ++s) {
    if (s == a.myseg) {
#pragma unroll
      for (int j = 0; j < 16; ++j) v[j] += t[j];
    } else {
      const int slot = partial_slot(a.c_lo + s, a.T, a.U, a.G, a.KC) * a.pmul + a.padd;
      const float* src = a.partials + (size_t)slot * a.N * kTileM;
#pragma unroll
      for (int j = 0; j < 16; ++j) v[j] += __ldcg(src + (size_t)(ch * 16 + j) * kTileM + a.r);
    }
  }
}

// Phases (one kernel instantiation each, so profiles attribute time per
// phase); kPhase also prunes the epilogues a phase cannot use.
enum Phase : int { PH_Z = 1, PH_ZLM = 2, PH_GH = 3, PH_SGH = 4, PH_FC2 = 5, PH_TABLE = 6, PH_ALL = 7 };

template <int kPhase>
__device__ __forceinline__ constexpr bool phase_has(int kind) {
  switch (kPhase) {
    case PH_Z: return kind == EPI_ZPROJ;
    case PH_ZLM: return kind == EPI_ZPROJ || kind == EPI_LMHEAD;
    case PH_GH: return kind == EPI_GH;
    case PH_SGH: return kind == EPI_SPROJ_MID || kind == EPI_GH;
    case PH_FC2: return kind == EPI_FC2_ARGMAX;
    case PH_TABLE: return kind == EPI_TABLE;
    case PH_ALL: return true;
  }
  return false;
}

// Pure-draft prefix tokens: the argmax over the vocab of the base logits at
// positions < npre, one 64-bit (value, index) word per row and position.  Out
// of line: it runs only for blocks with a pure-draft prefix.
template <typename T>
__device__ __noinline__ void prefix_argmax_chunk(unsigned long long* slots, int nslots, long long gn0, int nv, int kpos,
                                                 int npre, const T (&vals)[16], bool valid, uint32_t vocab_row,
                                                 int lane) {
  using IO = io<T>;
  for (int j = 0; j < 16 && j < nv; ++j) {
    const long long gn = gn0 + j;
    const int pos = (int)(gn % kpos);
    if (pos < npre) {  // uniform across the warp
      const float fv = IO::to_f(vals[j]);
      unsigned long long key = valid ? argmax_key(fv, vocab_row) : 0ull;
      key = warp_max_u64(key);
      if (lane == 0 && key) atomicMax(slots + (gn / kpos) * nslots + pos, key);
    }
  }
}

// Row stride of the staging area, in elements: 2-byte columns are padded by
// 64 bytes so that two consecutive columns start in opposite halves of the
// shared-memory banks.
template <typename T>
constexpr int kXStride = sizeof(T) == 2 ? kTileM + 32 : kTileM;

// Stage this thread's 16 column values of tile row r: S[j * kXStride + r].
// 2-byte values go as 32-bit words of two rows: lane pairs swap one value
// (even lanes write column j, odd lanes column j + 1), so each store covers
// 16 words of two padded columns without bank conflicts.
template <typename T>
__device__ __forceinline__ void stage_columns(T* S, const T (&vals)[16], int r) {
  if constexpr (sizeof(T) == 2) {
    const bool odd = (r & 1) != 0;
    uint32_t* S32 = reinterpret_cast<uint32_t*>(S);
#pragma unroll
    for (int j = 0; j < 16; j += 2) {
      const uint32_t mine0 = *reinterpret_cast<const uint16_t*>(&vals[j]);
      const uint32_t mine1 = *reinterpret_cast<const uint16_t*>(&vals[j + 1]);
      const uint32_t got = __shfl_xor_sync(0xFFFFFFFFu, odd ? mine0 : mine1, 1);
      const uint32_t word = odd ? (got | (mine1 << 16)) : (mine0 | (got << 16));
      const int col = odd ? j + 1 : j;
      S32[(col * kXStride<T> + (r & ~1)) >> 1] = word;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 16; ++j) S[j * kXStride<T> + r] = vals[j];
  }
}

template <typename T, int kPhase>
__device__ __forceinline__ void epilogue_tile(const GemvParams& p, const AccView& a, int kind, int row, bool valid,
                                              int q, int lane, unsigned long long* red, int ept) {
  using IO = io<T>;
  const int nchunks = p.N / 16;
  if ((phase_has<kPhase>(EPI_LMHEAD) || phase_has<kPhase>(EPI_ZPROJ) || phase_has<kPhase>(EPI_TABLE)) &&
      (kind == EPI_LMHEAD || kind == EPI_ZPROJ || kind == EPI_TABLE)) {
    float bias = 0.0f;
    if (valid) {
      if (kind == EPI_ZPROJ && p.fc1_bias) bias = IO::load((const T*)p.fc1_bias + row);
      if (kind == EPI_TABLE && p.b_ih) bias = IO::load((const T*)p.b_ih + row);
    }
    T* out;
    long long ld;
    if (kind == EPI_LMHEAD) {
      out = (T*)p.base_out;
      ld = p.base_out_ld;
    } else if (kind == EPI_ZPROJ) {
      out = (T*)p.z_out;
      ld = p.E;
    } else {
      out = (T*)p.table_out;
      ld = p.table_ld;
    }
    // Column n of the output is row-contiguous: the tile's 128 rows are
    // adjacent in memory, one X row apart from the next column.  Staged
    // through shared memory, each warp store covers 128 rows of one column
    // (4 elements per lane) instead of one element per lane, and a tile
    // touches each column's page once instead of four times.
    const bool xp = a.xpose != nullptr && (ld & 3) == 0 && (reinterpret_cast<uintptr_t>(out) & (4 * sizeof(T) - 1)) == 0;
    T* S = reinterpret_cast<T*>(a.xpose);
    const int w4 = (ept & 127) >> 5;  // warp within the warpgroup
    for (int ch = a.grp; ch < nchunks; ch += a.ngroups) {
      float v[16];
      acc_chunk(a, ch, v);
      T vals[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) vals[j] = IO::from_f(v[j] + bias);
      if (xp) {
        stage_columns<T>(S, vals, a.r);
      } else if (valid) {
#pragma unroll
        for (int j = 0; j < 16; ++j)
          if (ch * 16 + j < p.n_valid) out[((long long)p.n_off + ch * 16 + j) * ld + row] = vals[j];
      }
      if (kind == EPI_LMHEAD && p.npre > 0)
        prefix_argmax_chunk<T>(p.slots, p.nslots, (long long)p.n_off + ch * 16, p.n_valid - ch * 16, p.kpos, p.npre,
                               vals, valid, (uint32_t)(p.v_off + row), lane);
      if (xp) {
        named_bar_sync(a.bar, 128);
        const long long r0 = a.row0 + 4 * lane;  // first of this lane's four rows
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          const int j = w4 + 4 * jj;
          const int n = ch * 16 + j;
          if (n < p.n_valid) {
            T* dst = out + ((long long)p.n_off + n) * ld + r0;
            const T* src = S + j * kXStride<T> + 4 * lane;
            if (r0 + 3 < a.row_end) {
              store4<T>(dst, src);
            } else {
              for (int i = 0; i < 4; ++i)
                if (r0 + i < a.row_end) dst[i] = src[i];
            }
          }
        }
        named_bar_sync(a.bar, 128);
      }
    }
    return;
  }
  if (phase_has<kPhase>(EPI_GH) && kind == EPI_GH) {
    const float bias = (valid && p.b_hh) ? IO::load((const T*)p.b_hh + row) : 0.0f;
    for (int ch = 0; ch < nchunks; ++ch) {
      float v[16];
      acc_chunk(a, ch, v);
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int b = ch * 16 + j;
        if (b < p.B && valid) ((T*)p.gh_out)[(size_t)b * p.G3 + row] = IO::from_f(v[j] + bias);
      }
    }
    return;
  }
  if (phase_has<kPhase>(EPI_SPROJ_MID) && kind == EPI_SPROJ_MID) {
    for (int ch = 0; ch < nchunks; ++ch) {
      float v[16];
      acc_chunk(a, ch, v);
      // All z loads of the chunk first: the mid stores below could alias
      // them, so the compiler would otherwise serialise one L2 round trip
      // per batch row.
      float zv[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int b = ch * 16 + j;
        zv[j] = 0.0f;
        if (b < p.B && valid) {
          const size_t zrow = (size_t)b * p.z_rows_per_b + p.z_pos_off + p.t;
          zv[j] = IO::load((const T*)p.z_src + zrow * p.E + row);
        }
      }
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int b = ch * 16 + j;
        if (b < p.B && valid) {
          const T s_rounded = IO::from_f(v[j]);
          if (p.s_out) ((T*)p.s_out)[(size_t)b * p.E + row] = s_rounded;
          const float s = IO::to_f(s_rounded);
          const float z = zv[j];
          T hi, lo;
          if (p.middle == MID_SILU) {
            const float pre = z + s;
            const float mid = pre * sigmoidf_(pre);
            hi = IO::from_f(mid);
            lo = IO::from_f(mid - IO::to_f(hi));
          } else {
            // the PyTorch branch: mid = middle(z + s) in the weight dtype, one row
            hi = IO::from_f(middle_act(p.middle, IO::to_f(IO::from_f(z + s))));
            lo = IO::from_f(0.0f);
          }
          ((T*)p.mid_out)[(size_t)(2 * b) * p.E + row] = hi;
          ((T*)p.mid_out)[(size_t)(2 * b + 1) * p.E + row] = lo;
        }
      }
    }
    return;
  }
  if (phase_has<kPhase>(EPI_FC2_ARGMAX) && kind == EPI_FC2_ARGMAX) {
    const float bias = (valid && p.fc2_bias) ? IO::load((const T*)p.fc2_bias + row) : 0.0f;
    if (p.B > 4) {
      // One key per batch row in every lane, then a transposing butterfly:
      // each round halves the keys a lane holds, so 31 shuffles leave lane l
      // with the warp's maximum for batch row l (instead of 5 per row).
      // Base logit of batch row b: bptr[b * bstride], from the tile's staged
      // block in shared memory or from global memory.
      const T* bptr;
      long long bstride;
      if (a.bsm) {
        bptr = static_cast<const T*>(a.bsm) + a.r;
        bstride = kTileM;
      } else {
        bptr = (const T*)p.base_src + ((size_t)p.base_pos_off + p.t) * p.base_ld + p.base_voff + row;
        bstride = (long long)p.base_rows_per_b * p.base_ld;
      }
      unsigned long long k[kMaxBatch];
#pragma unroll
      for (int ch = 0; ch < kMaxBatch / 8; ++ch) {  // a 16-column chunk holds 8 rows (hi, lo)
        float v[16];
        if (ch < nchunks) acc_chunk(a, ch, v);
        float basev[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int b = ch * 8 + i;
          basev[i] = 0.0f;
          if (b < p.B && valid) basev[i] = IO::load(bptr + b * bstride);
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int b = ch * 8 + i;
          unsigned long long key = 0ull;
          if (b < p.B && valid && ch < nchunks) {
            float logit = v[2 * i] + v[2 * i + 1] + bias + basev[i];
            if (p.middle != MID_SILU)  // bias = F.linear(mid, fc2, b2); logits = base + bias, each in the dtype
              logit = IO::to_f(IO::from_f(IO::to_f(IO::from_f(v[2 * i] + v[2 * i + 1] + bias)) + basev[i]));
            key = argmax_key(logit, (uint32_t)(p.v_off + row));
          }
          k[b] = key;
        }
      }
#pragma unroll
      for (int o = kMaxBatch / 2; o >= 1; o >>= 1) {
        const bool up = (lane & o) != 0;
#pragma unroll
        for (int i = 0; i < o; ++i) {
          const unsigned long long send = up ? k[i] : k[i + o];
          const unsigned long long keep = up ? k[i + o] : k[i];
          const unsigned long long got = __shfl_xor_sync(0xFFFFFFFFu, send, o);
          k[i] = got > keep ? got : keep;
        }
      }
      red[q * kMaxBatch + lane] = k[0];
    } else {
      float v[16];
      acc_chunk(a, 0, v);  // 2B <= 8 columns
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        if (b < p.B) {
          unsigned long long key = 0ull;
          if (valid) {
            const size_t brow = (size_t)b * p.base_rows_per_b + p.base_pos_off + p.t;
            float logit = v[2 * b] + v[2 * b + 1];
            logit += bias;
            const float basev = IO::load((const T*)p.base_src + brow * p.base_ld + p.base_voff + row);
            if (p.middle != MID_SILU)  // bias = F.linear(mid, fc2, b2); logits = base + bias, each in the dtype
              logit = IO::to_f(IO::from_f(IO::to_f(IO::from_f(logit)) + basev));
            else
              logit += basev;
            key = argmax_key(logit, (uint32_t)(p.v_off + row));
          }
          key = warp_max_u64(key);
          if (lane == 0) red[q * kMaxBatch + b] = key;
        }
      }
    }
    named_bar_sync(a.bar, 128);
    if (ept < p.B) {
      unsigned long long k = red[ept];
#pragma unroll
      for (int w = 1; w < 4; ++w) {
        const unsigned long long o = red[w * kMaxBatch + ept];
        k = o > k ? o : k;
      }
      if (k) atomicMax(p.slots + (size_t)ept * p.nslots + p.npre + p.t, k);
    }
    named_bar_sync(a.bar, 128);
    return;
  }
}

// Called by the nthreads epilogue threads of every CTA once all of its tiles
// are finished.  The last CTA of the grid to get here sees every argmax word
// of the launch (atomicMax, fenced) and copies them to every rank's exchange
// buffer, then raises the flags.
__device__ __forceinline__ void publish_words(const GemvParams& p, int ept, volatile int* flag, int nthreads = 128) {
  const Exchange& x = p.xchg;
  named_bar_sync(1, nthreads);
  if (ept == 0) {
    __threadfence();
    const unsigned int old = atomicAdd(x.done + p.xslot0, 1u);
    const int last = old == gridDim.x - 1;
    if (last) {
      x.done[p.xslot0] = 0u;
      __threadfence();
    }
    *flag = last;
  }
  named_bar_sync(1, nthreads);
  if (!*flag) return;
  const unsigned long long seq = *x.seq;
  const int par = (int)(seq & 1ull);
  const int nsl = p.xslot1 - p.xslot0;
  const int n = x.world * nsl * x.B;
  for (int i = ept; i < n; i += nthreads) {
    const int j = i / (nsl * x.B);
    const int rem = i - j * nsl * x.B;
    const int slot = p.xslot0 + rem / x.B;
    const int b = rem - (rem / x.B) * x.B;
    const unsigned long long w = __ldcg(p.slots + (size_t)b * p.nslots + slot);
    __stcg(x.peer[j] + xchg_word(x, par, slot, x.rank, b), w);
  }
  __threadfence_system();
  named_bar_sync(1, nthreads);
  for (int i = ept; i < x.world * nsl; i += nthreads) {
    const int j = i / nsl;
    const int slot = p.xslot0 + (i - j * nsl);
    unsigned long long* f = x.peer[j] + xchg_flag(x, par, slot, x.rank);
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(f), "l"(seq) : "memory");
  }
}

// One-time relayout of a row-major weight matrix W [rows x K] (row stride ld
// elements, 2-byte elements) into 16 KB blocks, one per (128-row tile, 64-wide
// k-chunk), tile-major: block (t, kc) holds rows t*128 .. t*128+127, columns
// kc*64 .. kc*64+63, laid out exactly as a 128B-swizzled TMA box lands in
// shared memory (16-byte chunk j of row r at chunk j ^ (r & 7)); rows and
// columns past the matrix are zero.  A phase then streams each CTA's units as
// one contiguous run of 16 KB bulk copies.
__global__ void __launch_bounds__(256) pack_tiles_kernel(const uint16_t* __restrict__ w, long long rows, long long K,
                                                         long long ld, int KC, uint4* __restrict__ out) {
  const long long blk = blockIdx.x;  // = tile * KC + kc
  const long long tile = blk / KC;
  const int kc = (int)(blk - tile * KC);
  uint4* dst = out + blk * (kATileBytes / 16);
  for (int i = threadIdx.x; i < kTileM * 8; i += blockDim.x) {
    const int r = i >> 3, j = i & 7;
    const long long row = tile * kTileM + r;
    const long long col = (long long)kc * kChunkK + j * 8;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (row < rows) {
      const uint16_t* src = w + row * ld + col;
      if (col + 8 <= K && (reinterpret_cast<uintptr_t>(src) & 15) == 0) {
        v = *reinterpret_cast<const uint4*>(src);
      } else {
        uint16_t e[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) e[q] = (col + q < K) ? src[q] : (uint16_t)0;
        memcpy(&v, e, 16);
      }
    }
    dst[r * 8 + (j ^ (r & 7))] = v;
  }
}

// Sharded s / gh phase: once every CTA of this rank has written its tiles
// (mid hi/lo rows and gh of this rank's row slices), the last CTA raises this
// rank's flag for the step in every rank's exchange buffer.
__device__ __forceinline__ void publish_slices_done(const GemvParams& p, int ept, volatile int* flag) {
  const Exchange& x = p.xchg;
  named_bar_sync(1, 128);
  if (ept == 0) {
    __threadfence_system();  // this CTA's mid / gh stores, before it is counted
    const unsigned int old = atomicAdd(x.sdone + p.sflag_slot, 1u);
    const int last = old == gridDim.x - 1;
    if (last) {
      x.sdone[p.sflag_slot] = 0u;
      __threadfence_system();
    }
    *flag = last;
  }
  named_bar_sync(1, 128);
  if (!*flag) return;
  const unsigned long long seq = *x.seq;
  const int par = (int)(seq & 1ull);
  for (int j = ept; j < x.world; j += 128) {
    unsigned long long* f = x.peer[j] + x.sflag_off + ((size_t)par * x.nslots + p.sflag_slot) * x.world + x.rank;
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(f), "l"(seq) : "memory");
  }
}

// kEpiWarps = 8 (wide z / lm_head / table passes, one CTA per SM): two
// warpgroups read the accumulator's lane quadrants and split each tile's
// 16-column chunks between them.
// kPair (with kEpiWarps = 8): CTA pairs (clusters of 2) share each M = 256
// weight tile.  Each CTA loads its own 128 weight rows and half of the X rows;
// rank 0 issues the pair MMAs (cta_group::2) into both CTAs' TMEM and its
// commits release both CTAs' ring stages and accumulator slots; each CTA's
// epilogue finishes its own 128 rows, as a lone CTA does.  The pair reads X
// from shared memory once for both CTAs' rows.
template <typename T, int kPhase, int kEpiWarps = 4, bool kPair = false>
__global__ void __launch_bounds__((kEpiWarp0 + kEpiWarps) * 32, kEpiWarps == 4 ? 2 : 1)
    gemv_stream_kernel(const __grid_constant__ CUtensorMap tmA0, const __grid_constant__ CUtensorMap tmA1,
                       const __grid_constant__ CUtensorMap tmB, const GemvParams p) {
  static_assert(kEpiWarps == 4 || (kEpiWarps == 8 && (kPhase == PH_ZLM || kPhase == PH_Z || kPhase == PH_TABLE)),
                "two epilogue warpgroups only for the X-row-major output phases");
  static_assert(!kPair || kEpiWarps == 8, "CTA pairs run the wide passes only");
  constexpr int kEpiThreads = kEpiWarps * 32;
  constexpr int kGroups = kEpiWarps / 4;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = smem;
  uint8_t* tail = ring + (size_t)p.stages * p.stage_bytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(tail);
  uint64_t* empty = full + kMaxStages;
  uint64_t* accf = empty + kMaxStages;
  uint64_t* acce = accf + 2;
  uint64_t* drain = acce + 2;
  uint64_t* bfull = drain + 1;   // [2] base-logit tile landed (PH_FC2 staging)
  uint64_t* bempty = bfull + 2;  // [2] base-logit buffer read by the epilogue
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  volatile int* fin_flag = abort_flag + 1;
  // tail layout: [0, 512) barriers and flags, [512, 1024) counters, [1024, 2048) argmax reduction
  static_assert((2 * kMaxStages + 9) * 8 + 16 <= 512, "barrier block overflows its slot");
  static_assert(1024 + 4 * kMaxBatch * 8 <= kSmemTail, "reduction block overflows the tail");
  long long* issued = reinterpret_cast<long long*>(tail + 512);
  long long* consumed = issued + 1;
  long long* bissued = issued + 2;    // base tiles loaded by the producer
  long long* bconsumed = issued + 3;  // base tiles waited for by the epilogue
  uint8_t* bstage = tail + kSmemTail + p.xpose_bytes;  // [2][base_stage_bytes]
  unsigned long long* red = reinterpret_cast<unsigned long long*>(tail + 1024);  // [4][kMaxBatch]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // CTA pairs: the pair is the unit of the stream-K partition (c of G).
  const int rank = kPair ? (int)(blockIdx.x & 1u) : 0;
  const int G = kPair ? (int)(gridDim.x >> 1) : (int)gridDim.x;
  const int c = kPair ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const long long U = p.units;
  const long long u_begin = unit_begin(c, U, G);
  const long long u_end = unit_begin(c + 1, U, G);
  const int KC = p.KC;

  if (threadIdx.x == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&accf[s], 1);
      mbar_init(&acce[s], kPair ? 2 * kEpiThreads : kEpiThreads);  // pairs: both CTAs' epilogues, on rank 0
    }
    mbar_init(drain, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bfull[s], 1);
      mbar_init(&bempty[s], 1);
    }
    *abort_flag = 0;
    *fin_flag = 0;
    *issued = 0;
    *consumed = 0;
    *bissued = 0;
    *bconsumed = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmA0);
    if (p.nseg > 1 || p.base_stage_bytes) prefetch_tmap(&tmA1);
    prefetch_tmap(&tmB);
  }
  if (warp == 1) {
    if constexpr (kPair) {
      tmem_alloc_pair(tmem_holder, p.tmem_cols);  // warp 1 of both CTAs, together
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_holder, p.tmem_cols);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  if constexpr (kPair)
    cluster_sync_all();  // both CTAs' barriers exist before either signals the other's
  else
    __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  // Let the next phase's CTAs launch now; they only prefetch weights until
  // this grid has completed.
  pdl_launch_dependents();

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------ TMA producer
      const uint64_t pol_w = policy_evict_first();
      const uint64_t pol_keep = policy_evict_last();
      const uint64_t pol_x = policy_evict_last();
      const long long n_my = u_end - u_begin;
      const int pre = (int)(n_my < p.stages ? n_my : p.stages);
      // Unit u of this CTA's range is (tile, kc) = (u / KC, u % KC); the
      // loops below advance (tile, kc) and the ring position incrementally.
      auto load_a = [&](int stage, long long tile, int kc) {
        if constexpr (kPair) {
          const long long t128 = 2 * tile + rank;  // this CTA's 128 rows of the pair tile
          const uint32_t bar0 = smem_in_cta(&full[stage], 0);
          if (t128 >= p.tiles128) {  // past the last tile: a box of zeros (rows past segment 0's end)
            tma_load_2d_pair(ring + (size_t)stage * p.stage_bytes, &tmA0, bar0, kc * kChunkK,
                             (int)((p.seg[0].row_off / kTileM + p.seg[0].tiles) * kTileM), pol_w);
            return;
          }
          const bool s1 = t128 >= p.seg[0].tiles;
          const GemvSeg& sg = p.seg[s1 ? 1 : 0];
          const long long w_tile = (s1 ? t128 - p.seg[0].tiles : t128) + sg.row_off / kTileM;
          tma_load_2d_pair(ring + (size_t)stage * p.stage_bytes, s1 ? &tmA1 : &tmA0, bar0, kc * kChunkK,
                           (int)(w_tile * kTileM), pol_w);
          return;
        }
        const bool s1 = tile >= p.seg[0].tiles;
        const GemvSeg& sg = p.seg[s1 ? 1 : 0];
        const long long w_tile = (s1 ? tile - p.seg[0].tiles : tile) + sg.row_off / kTileM;
        const uint8_t* pk = p.packed[s1 ? 1 : 0];
        const uint64_t pol = p.w_keep[s1 ? 1 : 0] ? pol_keep : pol_w;
        if (pk) {
          bulk_load(ring + (size_t)stage * p.stage_bytes, pk + (size_t)(w_tile * KC + kc) * kATileBytes,
                    kATileBytes, &full[stage], pol);
        } else {
          tma_load_2d(ring + (size_t)stage * p.stage_bytes, s1 ? &tmA1 : &tmA0, &full[stage], kc * kChunkK,
                      (int)(w_tile * kTileM), pol);
        }
      };
      auto load_b = [&](int stage, int kc) {
        if constexpr (kPair)  // this CTA's half of the pass's X rows
          tma_load_2d_pair(ring + (size_t)stage * p.stage_bytes + kATileBytes, &tmB, smem_in_cta(&full[stage], 0),
                           kc * kChunkK, p.n_off + rank * p.b_box_rows, pol_x);
        else
          tma_load_2d(ring + (size_t)stage * p.stage_bytes + kATileBytes, &tmB, &full[stage], kc * kChunkK, p.n_off,
                      pol_x);
      };
      // The bytes a stage's full barrier waits for: pairs count both CTAs'
      // loads on rank 0's barrier, and only rank 0 posts them.
      auto expect_stage = [&](int stage) {
        if constexpr (kPair) {
          if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * (kATileBytes + p.b_bytes));
        } else {
          mbar_arrive_expect_tx(&full[stage], kATileBytes + p.b_bytes);
        }
      };
      const long long tile_begin = u_begin / KC;
      const int kc_begin = (int)(u_begin - tile_begin * KC);
      long long tile = tile_begin;
      int kc = kc_begin;
      // Weights first: they do not depend on the previous kernel.
      for (int i = 0; i < pre; ++i) {
        expect_stage(i);
        load_a(i, tile, kc);
        if (++kc == KC) {
          kc = 0;
          ++tile;
        }
      }
      // Then the weight tiles after the ring into L2: while this kernel waits
      // for the one before it (which may be latency-bound: a short launch, a
      // tail, the GRU cell), HBM keeps streaming this phase's weights.
      {
        const long long npf = n_my - pre < p.l2_prefetch_units ? n_my - pre : p.l2_prefetch_units;
        long long pt = tile;
        int pk = kc;
        for (long long i = 0; i < npf; ++i) {
          const bool s1 = pt >= p.seg[0].tiles;
          const GemvSeg& sg = p.seg[s1 ? 1 : 0];
          const long long w_tile = (s1 ? pt - p.seg[0].tiles : pt) + sg.row_off / kTileM;
          const uint8_t* pk_base = p.packed[s1 ? 1 : 0];
          if (pk_base)
            bulk_prefetch_l2(pk_base + (size_t)(w_tile * KC + pk) * kATileBytes, kATileBytes);
          else
            tma_prefetch_l2_2d(s1 ? &tmA1 : &tmA0, pk * kChunkK, (int)(w_tile * kTileM));
          if (++pk == KC) {
            pk = 0;
            ++pt;
          }
        }
      }
      pdl_wait_primary();
      fence_proxy_async_global();
      for (int i = 0, kb = kc_begin; i < pre; ++i) {
        load_b(i, kb);
        if (++kb == KC) kb = 0;
      }
      // Base-logit tiles (PH_FC2 staging), in tile order, in base_bufs
      // buffers: the base of every tile up to `upto` is loaded once its buffer
      // is free.  They come after the wait: the base logits may be written by
      // an earlier launch of the same call.  With two buffers the producer
      // may wait for one (the epilogue two tiles back frees it).  With one it
      // must not: the buffer is freed by the epilogue of the tile before,
      // whose MMAs need the weight stages the producer has yet to issue, so
      // it only tests the buffer between stages and waits once its stages
      // are all issued.
      long long btile = tile_begin;
      const long long tile_last = n_my > 0 ? (u_end - 1) / KC : tile_begin - 1;  // no units: no base tiles
      const int nb = p.base_bufs;
      auto base_upto = [&](long long upto, bool block) -> bool {
        if (!p.base_stage_bytes) return true;
        for (; btile <= upto && btile <= tile_last; ++btile) {
          const long long n = btile - tile_begin;
          const int bs = (int)(n % nb);
          const uint32_t par = (uint32_t)(((n / nb) & 1) ^ 1);
          if (block) {
            if (!mbar_wait_bounded(&bempty[bs], par, abort_flag)) return false;
          } else if (!mbar_test_wait(&bempty[bs], par)) {
            return true;  // still in use: try again after the next stage
          }
          mbar_arrive_expect_tx(&bfull[bs], p.base_stage_bytes);
          tma_load_3d(bstage + (size_t)bs * p.base_stage_bytes, &tmA1, &bfull[bs],
                      (int)(p.base_voff + btile * kTileM), p.base_pos_off + p.t, 0);
          *bissued = n + 1;
        }
        return true;
      };
      bool ok = nb > 1 ? base_upto((u_begin + (pre > 0 ? pre - 1 : 0)) / KC, true)
                       : base_upto(tile_begin, true);  // the one buffer starts free
      int stage = pre == p.stages ? 0 : pre;
      uint32_t parity = pre == p.stages ? 1u : 0u;
      long long it = pre;
      for (; ok && it < n_my; ++it) {
        if (!base_upto(tile, nb > 1)) break;
        if (!mbar_wait_bounded(&empty[stage], parity ^ 1u, abort_flag)) break;
        expect_stage(stage);
        load_a(stage, tile, kc);
        load_b(stage, kc);
        if (++kc == KC) {
          kc = 0;
          ++tile;
        }
        if (++stage == p.stages) {
          stage = 0;
          parity ^= 1u;
        }
      }
      *issued = it;
      if (ok && it == n_my) base_upto(tile_last, true);  // one buffer: the bases not issued yet
    }
  } else if (warp == 1) {
    pdl_wait_primary();
    if (lane == 0 && rank == 0) {
      // ------------------------------------------------ MMA issuer
      long long u = u_begin;
      long long it = 0;
      int stage = 0;
      uint32_t parity = 0;
      int acc_it = 0;
      bool ok = true;
      while (ok && u < u_end) {
        const long long tile = u / KC;
        const int kc0 = (int)(u % KC);
        const long long left = u_end - u;
        const int kc1 = (int)((KC - kc0) < left ? KC : kc0 + left);
        const int slot = acc_it % p.acc_slots;
        const uint32_t use = (uint32_t)(acc_it / p.acc_slots);
        if (!mbar_wait_bounded(&acce[slot], (use & 1u) ^ 1u, abort_flag)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + (uint32_t)(slot * p.N * p.nacc);
        for (int kc = kc0; kc < kc1; ++kc, ++it) {
          if (!mbar_wait_bounded(&full[stage], parity, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(ring + (size_t)stage * p.stage_bytes);
          const uint64_t adesc = smem_desc_k_sw128(a_addr);
          const uint64_t bdesc = smem_desc_k_sw128(a_addr + kATileBytes);
          // Consecutive K-steps go to different accumulators so that the
          // tensor pipe overlaps them instead of chaining on one accumulator.
#pragma unroll
          for (int k = 0; k < kChunkK / 16; ++k) {
            const int ks = (kc - kc0) * (kChunkK / 16) + k;
            const int acc = ks % p.nacc;
            if constexpr (kPair)
              mma_f16_ss_pair(d + (uint32_t)(acc * p.N), adesc + 2 * k, bdesc + 2 * k, p.idesc, ks >= p.nacc ? 1u : 0u);
            else
              mma_f16_ss(d + (uint32_t)(acc * p.N), adesc + 2 * k, bdesc + 2 * k, p.idesc, ks >= p.nacc ? 1u : 0u);
          }
          if constexpr (kPair) {  // the stage is free in both CTAs
            mma_commit_pair(smem_in_cta(&empty[stage], 0));
            mma_commit_pair(smem_in_cta(&empty[stage], 1));
          } else {
            mma_commit(&empty[stage]);
          }
          if (++stage == p.stages) {
            stage = 0;
            parity ^= 1u;
          }
        }
        if (!ok) break;
        if constexpr (kPair) {  // both CTAs' accumulators are ready
          mma_commit_pair(smem_in_cta(&accf[slot], 0));
          mma_commit_pair(smem_in_cta(&accf[slot], 1));
        } else {
          mma_commit(&accf[slot]);
        }
        ++acc_it;
        u += kc1 - kc0;
        (void)tile;
      }
      *consumed = it;
    }
  } else {
    // -------------------------------------------------- epilogue (warps 2 .. 2 + kEpiWarps - 1)
    pdl_wait_primary();
    const int ept = threadIdx.x - kEpiWarp0 * 32;  // 0 .. kEpiThreads - 1
    const int grp = ept >> 7;                       // warpgroup
    const int q = warp & 3;                         // TMEM lane quadrant of this warp
    const int r = q * 32 + lane;                    // row within the tile
    long long u = u_begin;
    int acc_it = 0;
    while (u < u_end) {
      const long long tile = u / KC;
      const int kc0 = (int)(u % KC);
      const long long left = u_end - u;
      const int kc1 = (int)((KC - kc0) < left ? KC : kc0 + left);
      const int slot = acc_it % p.acc_slots;
      const uint32_t use = (uint32_t)(acc_it / p.acc_slots);
      const bool got = mbar_wait_bounded(&accf[slot], use & 1u, abort_flag);
      if (!named_bar_and(1, kEpiThreads, got)) break;
      tc_fence_after();

      // The 128-row tile this CTA finishes (pairs: its half of the pair tile).
      const long long t128 = kPair ? 2 * tile + rank : tile;
      if (kPair && t128 >= p.tiles128) {  // the empty half of a last pair tile: nothing to finish
        tc_fence_before();
        mbar_arrive_cluster(smem_in_cta(&acce[slot], 0));
        ++acc_it;
        u += kc1 - kc0;
        continue;
      }
      const bool s1 = t128 >= p.seg[0].tiles;
      const GemvSeg& sg = p.seg[s1 ? 1 : 0];
      const int local_row = (int)((s1 ? t128 - p.seg[0].tiles : t128) * kTileM) + r;
      const bool valid = local_row < sg.rows;
      const int row = sg.row_off + local_row;

      AccView a;
      a.taddr = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(slot * p.N * p.nacc);
      a.nacc = p.nacc;
      a.bar = kGroups > 1 ? 2 + grp : 1;
      a.xpose = p.xpose_bytes ? tail + kSmemTail + (size_t)grp * kXposeBytes : nullptr;
      a.grp = grp;
      a.ngroups = kGroups;
      a.row0 = row - r;
      a.row_end = (long long)sg.row_off + sg.rows;
      a.combine = false;
      a.nseg = 1;
      a.myseg = 0;
      a.c_lo = c;
      a.T = tile;
      a.partials = p.partials;
      a.N = p.N;
      a.r = r;
      a.U = U;
      a.G = G;
      a.KC = KC;
      a.bsm = nullptr;
      a.pmul = kPair ? 2 : 1;
      a.padd = rank;
      int bslot = 0;
      if constexpr (kPhase == PH_FC2) {
        if (p.base_stage_bytes) {
          // every tile's base load is waited for (in order), finished here or not
          const long long n = tile - u_begin / KC;
          bslot = (int)(n % p.base_bufs);
          const bool landed = mbar_wait_bounded(&bfull[bslot], (uint32_t)((n / p.base_bufs) & 1), abort_flag);
          if (!named_bar_and(1, kEpiThreads, landed)) break;
          if (ept == 0) *bconsumed = n + 1;
          a.bsm = bstage + (size_t)bslot * p.base_stage_bytes;
        }
      }

      bool finish = true;
      if (kc0 > 0 || kc1 < KC) {
        // Split tile: publish this CTA's partial; the last segment to arrive finishes.
        const int c_lo = cta_of_unit(tile * KC, U, G);
        const int c_hi = cta_of_unit(tile * KC + KC - 1, U, G);
        a.nseg = c_hi - c_lo + 1;
        a.myseg = c - c_lo;
        a.c_lo = c_lo;
        float* mine = p.partials + (size_t)(partial_slot(c, tile, U, G, KC) * a.pmul + a.padd) * p.N * kTileM;
        for (int ch = grp; ch < p.N / 16; ch += kGroups) {
          float v[16];
          acc_local(a, ch, v);
#pragma unroll
          for (int j = 0; j < 16; ++j) __stcg(mine + (size_t)(ch * 16 + j) * kTileM + r, v[j]);
        }
        __threadfence();
        named_bar_sync(1, kEpiThreads);
        if (ept == 0) {
          const unsigned int old = atomicAdd(p.tile_counters + t128, 1u);
          const int last = (old == (unsigned int)(a.nseg - 1)) ? 1 : 0;
          if (last) {
            p.tile_counters[t128] = 0u;  // ready for the next phase
            __threadfence();
          }
          *fin_flag = last;
        }
        named_bar_sync(1, kEpiThreads);
        finish = *fin_flag != 0;
        if (finish) {
          __threadfence();
          a.combine = true;
        }
      }
      if (finish) epilogue_tile<T, kPhase>(p, a, sg.kind, row, valid, q, lane, red, ept);
      if constexpr (kPhase == PH_FC2) {
        if (p.base_stage_bytes) {
          named_bar_sync(1, kEpiThreads);  // all reads of this base buffer done
          if (ept == 0) mbar_arrive(&bempty[bslot]);
        }
      }

      tc_fence_before();
      if constexpr (kPair)
        mbar_arrive_cluster(smem_in_cta(&acce[slot], 0));  // rank 0's MMA issuer waits for both CTAs
      else
        mbar_arrive(&acce[slot]);
      ++acc_it;
      u += kc1 - kc0;
    }
    if constexpr (kPhase == PH_FC2 || kPhase == PH_ZLM) {
      // All 128 threads decide together whether to publish (publish_words
      // contains named barriers).
      if (p.xchg.world > 1 && p.xslot1 > p.xslot0 && named_bar_and(1, kEpiThreads, *abort_flag == 0))
        publish_words(p, ept, fin_flag, kEpiThreads);
    }
    if constexpr (kPhase == PH_SGH) {
      if (p.xchg.world > 1 && p.sflag_slot >= 0 && named_bar_and(1, kEpiThreads, *abort_flag == 0))
        publish_slices_done(p, ept, fin_flag);
    }
    if constexpr (kPhase == PH_FC2) {
      if (p.fused_cell) {
        // Every CTA's argmax words are final once all have arrived; then each
        // CTA runs its share of the GRU step (a CTA that gave up arrives
        // without waiting, so that the others are not held).
        named_bar_sync(1, kEpiThreads);
        if (ept == 0) {
          const bool aborted = *abort_flag != 0;
          const bool ok = grid_barrier(p.gbar, gridDim.x, !aborted);
          if (!ok) atomicOr(p.status, 1u /* DD_STATUS_TIMEOUT */);
          *fin_flag = ok && !aborted;
        }
        named_bar_sync(1, kEpiThreads);
        if (*fin_flag) {
          const int n = p.cell.B * (p.cell.G / 8);
          for (int idx = c * 128 + ept; idx < n; idx += G * 128) cell_apply<T>(p.cell, idx);
        }
      }
    }
  }

  __syncthreads();
  if constexpr (kPair) {
    // Rank 0's MMAs read both CTAs' shared memory and write both CTAs' TMEM,
    // and both epilogues arrive on rank 0's barriers: neither CTA releases
    // anything before the other is done.
    if (*abort_flag && rank == 0 && warp == 1 && lane == 0) {
      mma_commit_pair(smem_in_cta(drain, 0));
      wait_ns(drain, 0, 100ull * 1000 * 1000);
    }
    cluster_sync_all();
    // After a timed-out wait in either CTA: both CTAs' loads count on rank
    // 0's full barriers, so rank 0 lets every stage either CTA issued land.
    if (rank == 0 && warp == 0 && lane == 0) {
      const bool peer_abort = ld_cluster_u32(smem_in_cta((const void*)abort_flag, 1)) != 0;
      if (*abort_flag || peer_abort) {
        const long long peer_issued = ld_cluster_s64(smem_in_cta(issued, 1));
        const long long upto = *issued > peer_issued ? *issued : peer_issued;
        for (long long it = *consumed; it < upto; ++it)
          wait_ns(&full[it % p.stages], (uint32_t)((it / p.stages) & 1), 100ull * 1000 * 1000);
      }
    }
    if (*abort_flag && threadIdx.x == 0) atomicOr(p.status, 1u /* DD_STATUS_TIMEOUT */);
    cluster_sync_all();
  } else {
    if (*abort_flag) {
      // Unwind after a timed-out wait: let in-flight MMAs and TMA loads land
      // before the shared memory and TMEM are released.
      if (warp == 1 && lane == 0) {
        mma_commit(drain);
        wait_ns(drain, 0, 100ull * 1000 * 1000);
      }
      if (warp == 0 && lane == 0) {
        for (long long it = *consumed; it < *issued; ++it)
          wait_ns(&full[it % p.stages], (uint32_t)((it / p.stages) & 1), 100ull * 1000 * 1000);
        for (long long n = *bconsumed; n < *bissued; ++n)
          wait_ns(&bfull[n % p.base_bufs], (uint32_t)((n / p.base_bufs) & 1), 100ull * 1000 * 1000);
      }
      if (threadIdx.x == 0) atomicOr(p.status, 1u /* DD_STATUS_TIMEOUT */);
      __syncthreads();
    }
  }
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    if constexpr (kPair)
      tmem_dealloc_pair(tmem_base, p.tmem_cols);
    else
      tmem_dealloc(tmem_base, p.tmem_cols);
  }
}

}  // namespace dd
