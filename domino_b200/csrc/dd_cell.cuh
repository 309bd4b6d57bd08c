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
// the words and the counter for the next call.
constexpr int kVerifyThreads = 256;
constexpr int kVerifyChunk = 32768;
constexpr int kMaxVerifyK1 = 64;  // positions per row (the handle's word buffer holds B x 64)  // vocab entries per CTA: 16 16-byte loads per thread in flight

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
  __device__ __forceinline__ void see(float x, int idx) {
    const bool take = (x > v) || (x != x && v == v) || i < 0;
    v = take ? x : v;
    i = take ? idx : i;
  }
  __device__ __forceinline__ unsigned long long key() const {
    return i < 0 ? 0ull : argmax_key(v, (uint32_t)i);
  }
};

template <typename L>
__global__ void __launch_bounds__(kVerifyThreads) verify_accept_kernel(const L* logits, int V, int B, int K1,
                                                                      const int64_t* verify, int64_t* posterior,
                                                                      int32_t* accept, int64_t* bonus,
                                                                      unsigned long long* words,
                                                                      unsigned int* done, unsigned int* status) {
  pdl_launch_dependents();
  pdl_wait_primary();
  __shared__ unsigned long long red[kVerifyThreads / 32];
  __shared__ int last;
  const int row = blockIdx.y;
  const int v0 = blockIdx.x * kVerifyChunk;
  const int v1 = min(V, v0 + kVerifyChunk);
  const L* src = logits + (size_t)row * V;
  // 16-byte loads over the aligned middle of [v0, v1); rows of odd length
  // start anywhere, so the first `head` elements and the tail go one by one.
  // Each thread sees its indices in increasing order: head, vectors, tail.
  constexpr int kVec = 16 / (int)sizeof(L);
  const int head = min(v1 - v0, (int)(((16u - (reinterpret_cast<uintptr_t>(src + v0) & 15u)) & 15u) / sizeof(L)));
  const int nvec = (v1 - v0 - head) / kVec;
  const int vtail = v0 + head + nvec * kVec;
  ArgmaxRun run;
  if ((int)threadIdx.x < head) run.see(logit_f<L>(src[v0 + threadIdx.x]), v0 + threadIdx.x);
  const uint4* vsrc = reinterpret_cast<const uint4*>(src + v0 + head);
#pragma unroll 4
  for (int i = threadIdx.x; i < nvec; i += kVerifyThreads) {
    const uint4 raw = __ldcs(vsrc + i);  // read once: do not keep it in L2
    const L* e = reinterpret_cast<const L*>(&raw);
    const int vb = v0 + head + i * kVec;
#pragma unroll
    for (int j = 0; j < kVec; ++j) run.see(logit_f<L>(e[j]), vb + j);
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
