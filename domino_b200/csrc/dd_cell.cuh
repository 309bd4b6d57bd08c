// dd_cell.cuh -- the small kernels between the weight-streaming phases:
//   cell_kernel    picks the step's token (argmax word or a given id), writes
//                  it out, gathers gi = table[token] and runs the GRU cell
//                  h' = (1 - z) n + z h in fp32 (code/kernel/domino.py:172-226,
//                  with gi from the embed @ W_ih^T table, domino.py:418);
//   accept_kernel  greedy prefix acceptance (code/dflash.py:472-485).
#pragma once

#include "dd_gemv.cuh"

namespace dd {

template <typename T>
__global__ void __launch_bounds__(128) cell_kernel(const CellParams p) {
  pdl_launch_dependents();
  pdl_wait_primary();
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= p.B * (p.G / 8)) return;
  cell_apply<T>(p, idx);
}

// accept[b] = number of leading draft tokens equal to the target's greedy
// tokens: (verify[:, 1:] == posterior[:, :-1]).cumprod(1).sum(1);
// bonus[b] = posterior[b, accept[b]].
__global__ void __launch_bounds__(128) accept_kernel(const int64_t* verify, const int64_t* posterior, int B, int K1,
                                                     int32_t* accept, int64_t* bonus) {
  pdl_launch_dependents();
  pdl_wait_primary();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  const int64_t* v = verify + (size_t)b * K1;
  const int64_t* q = posterior + (size_t)b * K1;
  int a = 0;
  while (a < K1 - 1 && v[a + 1] == q[a]) ++a;
  accept[b] = a;
  bonus[b] = q[a];
}

// Sharded s / gh phase, gather side: wait (bounded) until every other rank
// has raised its flag for step `slot`, then copy that rank's column slices of
// mid (rows 0 .. mid_rows-1, columns [e0[j], e1[j])) and gh (rows 0 .. B-1,
// columns [g0[j], g1[j])) from its buffers (peer loads over NVLink) into
// this rank's.  Slice bounds are multiples of 128 elements (16-byte vectors).
struct GatherParams {
  Exchange xchg;
  const unsigned long long* xbuf;  // this rank's exchange buffer (flags)
  int slot;
  int mid_rows, E, G3, B;
  int e0[kMaxRanks], e1[kMaxRanks], g0[kMaxRanks], g1[kMaxRanks];
  int with_gh;
  unsigned int* status;
};

__global__ void __launch_bounds__(256) gather_slices_kernel(const GatherParams p) {
  pdl_launch_dependents();
  pdl_wait_primary();
  const Exchange& x = p.xchg;
  const unsigned long long seq = *x.seq;
  const int par = (int)(seq & 1ull);
  // vectors of 8 elements per (peer, row, column-chunk)
  long long total = 0;
  long long mid_n[kMaxRanks], gh_n[kMaxRanks];
  for (int j = 0; j < x.world; ++j) {
    mid_n[j] = (j == x.rank) ? 0 : (long long)p.mid_rows * ((p.e1[j] - p.e0[j]) / 8);
    gh_n[j] = (j == x.rank || !p.with_gh) ? 0 : (long long)p.B * ((p.g1[j] - p.g0[j]) / 8);
    total += mid_n[j] + gh_n[j];
  }
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    long long k = i;
    int j = 0;
    while (k >= mid_n[j] + gh_n[j]) {
      k -= mid_n[j] + gh_n[j];
      ++j;
    }
    // rank j's slices are complete once its flag for this step is raised
    const unsigned long long* f = p.xbuf + x.sflag_off + ((size_t)par * x.nslots + p.slot) * x.world + j;
    const uint64_t t0 = globaltimer_ns();
    bool ok = true;
    while (true) {
      unsigned long long v;
      asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(f) : "memory");
      if (v == seq) break;
      if (globaltimer_ns() - t0 > x.timeout_ns) {
        atomicOr(p.status, 1u /* DD_STATUS_TIMEOUT */);
        ok = false;
        break;
      }
      __nanosleep(64);
    }
    if (!ok) continue;
    const uint8_t* src_base = reinterpret_cast<const uint8_t*>(x.peer[j]);
    uint8_t* dst_base = reinterpret_cast<uint8_t*>(const_cast<unsigned long long*>(p.xbuf));
    size_t off;
    if (k < mid_n[j]) {
      const int per_row = (p.e1[j] - p.e0[j]) / 8;
      const long long row = k / per_row;
      const int c = (int)(k - row * per_row);
      off = x.mid_off + ((size_t)row * p.E + p.e0[j] + c * 8) * 2;
    } else {
      k -= mid_n[j];
      const int per_row = (p.g1[j] - p.g0[j]) / 8;
      const long long row = k / per_row;
      const int c = (int)(k - row * per_row);
      off = x.gh_off + ((size_t)row * p.G3 + p.g0[j] + c * 8) * 2;
    }
    const uint4 v = __ldcv(reinterpret_cast<const uint4*>(src_base + off));
    *reinterpret_cast<uint4*>(dst_base + off) = v;
  }
}

// Greedy verify fused with acceptance (code/dflash.py:472-485):
// posterior[b, j] = argmax_v logits[b, j, v] (lowest index on ties) and the
// acceptance of verify[b, :] against it, in one pass over the logits.
// Grid (chunks, B * K1): each CTA reduces one chunk of one row to a packed
// (value, index) word and atomicMax-es it into words[row]; the last CTA to
// finish (done counter) decodes all rows, runs the prefix match, and clears
// the words and the counter for the next call.  The host sizes the chunk so
// that the grid is one wave of resident CTAs where the rows allow it.
constexpr int kVerifyThreads = 256;
constexpr int kVerifyGroup = 4;    // 16-byte vectors a thread reduces at a time
constexpr int kMaxVerifyK1 = 64;   // positions per row (the handle's word buffer holds B x 64)

template <typename L>
__device__ __forceinline__ float logit_f(L v);
template <>
__device__ __forceinline__ float logit_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ float logit_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <>
__device__ __forceinline__ float logit_f<__half>(__half v) { return __half2float(v); }

// Running (value, index) argmax over increasing indices: a strictly larger
// value replaces the best, so the first of equal maxima stays, and a NaN
// replaces a number but not an earlier NaN (torch.argmax's order).
struct ArgmaxRun {
  float v = -INFINITY;
  int i = -1;
  __device__ __forceinline__ bool beaten_by(float x) const { return (x > v) || (x != x && v == v) || i < 0; }
  __device__ __forceinline__ void see(float x, int idx) {
    const bool take = beaten_by(x);
    v = take ? x : v;
    i = take ? idx : i;
  }
  // -0 and +0 compare equal for torch.argmax, so the word of a zero maximum
  // carries +0: across threads the lower index then wins, as in torch.
  __device__ __forceinline__ unsigned long long key() const {
    return i < 0 ? 0ull : argmax_key(v == 0.0f ? 0.0f : v, (uint32_t)i);
  }
};

// Packed arithmetic on the 32-bit words of a logits vector: two bf16 / fp16
// logits or one fp32 logit per word, element 0 in the low half.
//   wmax   NaN-propagating max of two words, lane by lane;
//   top    the largest value of a word as fp32 (NaN if either is NaN);
//   bcast  a word holding the value x (exactly representable) in every lane;
//   match  per-lane mask of the lanes equal to the broadcast value (IEEE
//          equality, so -0 matches +0), or of the NaN lanes when `nan`.
template <typename L>
struct VerifyWords;
template <>
struct VerifyWords<__nv_bfloat16> {
  static constexpr int kPer = 2;
  static __device__ __forceinline__ uint32_t wmax(uint32_t a, uint32_t b) {
    const __nv_bfloat162 r = __hmax2_nan(*reinterpret_cast<const __nv_bfloat162*>(&a),
                                         *reinterpret_cast<const __nv_bfloat162*>(&b));
    return *reinterpret_cast<const uint32_t*>(&r);
  }
  static __device__ __forceinline__ float top(uint32_t w) {
    const __nv_bfloat162 p = *reinterpret_cast<const __nv_bfloat162*>(&w);
    return __bfloat162float(__hmax_nan(p.x, p.y));
  }
  static __device__ __forceinline__ uint32_t bcast(float x) {
    const __nv_bfloat162 p = __float2bfloat162_rn(x);
    return *reinterpret_cast<const uint32_t*>(&p);
  }
  static __device__ __forceinline__ uint32_t match(uint32_t w, uint32_t m, bool nan) {
    return nan ? __vcmpgtu2(w & 0x7FFF7FFFu, 0x7F807F80u)
               : __heq2_mask(*reinterpret_cast<const __nv_bfloat162*>(&w), *reinterpret_cast<const __nv_bfloat162*>(&m));
  }
};
template <>
struct VerifyWords<__half> {
  static constexpr int kPer = 2;
  static __device__ __forceinline__ uint32_t wmax(uint32_t a, uint32_t b) {
    const __half2 r = __hmax2_nan(*reinterpret_cast<const __half2*>(&a), *reinterpret_cast<const __half2*>(&b));
    return *reinterpret_cast<const uint32_t*>(&r);
  }
  static __device__ __forceinline__ float top(uint32_t w) {
    const __half2 p = *reinterpret_cast<const __half2*>(&w);
    return __half2float(__hmax_nan(p.x, p.y));
  }
  static __device__ __forceinline__ uint32_t bcast(float x) {
    const __half2 p = __float2half2_rn(x);
    return *reinterpret_cast<const uint32_t*>(&p);
  }
  static __device__ __forceinline__ uint32_t match(uint32_t w, uint32_t m, bool nan) {
    return nan ? __vcmpgtu2(w & 0x7FFF7FFFu, 0x7C007C00u)
               : __heq2_mask(*reinterpret_cast<const __half2*>(&w), *reinterpret_cast<const __half2*>(&m));
  }
};
template <>
struct VerifyWords<float> {
  static constexpr int kPer = 1;
  static __device__ __forceinline__ uint32_t wmax(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("max.NaN.f32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
  }
  static __device__ __forceinline__ float top(uint32_t w) { return __uint_as_float(w); }
  static __device__ __forceinline__ uint32_t bcast(float x) { return __float_as_uint(x); }
  static __device__ __forceinline__ uint32_t match(uint32_t w, uint32_t m, bool nan) {
    const float x = __uint_as_float(w);
    return (nan ? x != x : x == __uint_as_float(m)) ? 1u : 0u;
  }
};

template <typename L>
__global__ void __launch_bounds__(kVerifyThreads) verify_accept_kernel(const L* logits, int V, int chunk, int B, int K1,
                                                                      const int64_t* verify, int64_t* posterior,
                                                                      int32_t* accept, int64_t* bonus,
                                                                      unsigned long long* words,
                                                                      unsigned int* done, unsigned int* status) {
  using W = VerifyWords<L>;
  constexpr int kVec = 16 / (int)sizeof(L);       // logits per 16-byte vector
  constexpr int kWords = 4 * kVerifyGroup;        // 32-bit words per group
  pdl_launch_dependents();
  pdl_wait_primary();
  __shared__ unsigned long long red[kVerifyThreads / 32];
  __shared__ int last;
  const int row = blockIdx.y;
  const int v0 = blockIdx.x * chunk;
  const int v1 = min(V, v0 + chunk);
  const L* src = logits + (size_t)row * V;
  // 16-byte loads over the aligned middle of [v0, v1); rows of odd length
  // start anywhere, so the first `head` elements and the tail go one by one.
  // Each thread sees its indices in increasing order: head, groups, tail.
  const int head = min(v1 - v0, (int)(((16u - (reinterpret_cast<uintptr_t>(src + v0) & 15u)) & 15u) / sizeof(L)));
  const int nvec = (v1 - v0 - head) / kVec;
  const int vbase = v0 + head;
  const int vtail = vbase + nvec * kVec;
  ArgmaxRun run;
  if ((int)threadIdx.x < head) run.see(logit_f<L>(src[v0 + threadIdx.x]), v0 + threadIdx.x);
  const uint4* vsrc = reinterpret_cast<const uint4*>(src + vbase);
  // Groups: vectors t, t + 256, t + 512, t + 768 (coalesced across the CTA).
  // The group's maximum comes from a tree of packed NaN-propagating maxima;
  // only a group that beats the running best is searched for the first
  // position holding that maximum.  In the last group of a thread the vectors
  // past the end are copies of its first vector: a copy never holds a value
  // that the original, at a lower index, does not hold first.
  constexpr int kStride = kVerifyThreads * kVerifyGroup;
  for (int i = threadIdx.x; i < nvec; i += kStride) {
    uint32_t w[kWords];
    const uint4 first = __ldcs(vsrc + i);  // read once: do not keep it in L2
    w[0] = first.x; w[1] = first.y; w[2] = first.z; w[3] = first.w;
#pragma unroll
    for (int j = 1; j < kVerifyGroup; ++j) {
      const int idx = i + j * kVerifyThreads;
      const uint4 raw = idx < nvec ? __ldcs(vsrc + idx) : first;
      w[4 * j + 0] = raw.x; w[4 * j + 1] = raw.y; w[4 * j + 2] = raw.z; w[4 * j + 3] = raw.w;
    }
    uint32_t m[kWords / 2];
#pragma unroll
    for (int k = 0; k < kWords / 2; ++k) m[k] = W::wmax(w[2 * k], w[2 * k + 1]);
#pragma unroll
    for (int s = kWords / 4; s >= 1; s >>= 1)
#pragma unroll
      for (int k = 0; k < s; ++k) m[k] = W::wmax(m[k], m[k + s]);
    const float gm = W::top(m[0]);
    if (run.beaten_by(gm)) {
      const bool nan = gm != gm;
      const uint32_t mb = W::bcast(gm);
      int pos = 0;  // first lane (in index order) of the group holding gm
#pragma unroll
      for (int k = kWords - 1; k >= 0; --k) {
        const uint32_t mk = W::match(w[k], mb, nan);
        if (mk) pos = k * W::kPer + ((W::kPer == 2 && !(mk & 0xFFFFu)) ? 1 : 0);
      }
      const int j = pos / kVec, e = pos - j * kVec;
      run.v = gm;
      run.i = vbase + (i + j * kVerifyThreads) * kVec + e;
    }
  }
  for (int v = vtail + threadIdx.x; v < v1; v += kVerifyThreads) run.see(logit_f<L>(src[v]), v);
  unsigned long long best = run.key();
  best = warp_max_u64(best);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long k = red[0];
    for (int w = 1; w < kVerifyThreads / 32; ++w) k = red[w] > k ? red[w] : k;
    if (k) atomicMax(words + row, k);
    __threadfence();
    const unsigned int total = gridDim.x * gridDim.y;
    last = atomicAdd(done, 1u) == total - 1;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  // The last CTA: one word per thread decoded into the posterior (and shared
  // memory), then the prefix match of every row from shared memory.
  __shared__ int32_t post[kMaxBatch * kMaxVerifyK1];
  __shared__ int64_t ver[kMaxBatch * kMaxVerifyK1];
  const int n = B * K1;
  for (int i = threadIdx.x; i < n; i += kVerifyThreads) {
    const unsigned long long k = __ldcg(words + i);
    if (!k) atomicOr(status, 4u /* DD_STATUS_NO_ARGMAX */);
    const int32_t tok = k ? (int32_t)argmax_key_index(k) : 0;
    post[i] = tok;
    ver[i] = verify[i];
    posterior[i] = tok;
    words[i] = 0ull;  // ready for the next call
  }
  __syncthreads();
  for (int b = threadIdx.x; b < B; b += kVerifyThreads) {
    int a = 0;
    while (a + 1 < K1 && ver[b * K1 + a + 1] == (int64_t)post[b * K1 + a]) ++a;
    accept[b] = a;
    bonus[b] = post[b * K1 + a];
  }
  if (threadIdx.x == 0) *done = 0u;
}

}  // namespace dd
