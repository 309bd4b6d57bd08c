// dd_cell_core.cuh -- the GRU step of one rollout step, shared by the cell
// kernel (dd_cell.cuh) and the fc2 launch that runs it in its tail
// (dd_gemv.cuh): the argmax word -> token, gi = table[token] and the fused
// cell h' = (1 - z) n + z h in fp32 (code/kernel/domino.py:172-226, with gi
// from the embed @ W_ih^T table, domino.py:418), plus the argmax-word
// exchange of vocab-sharded ranks.
#pragma once

#include "dd_ptx.cuh"

namespace dd {

constexpr int kMaxRanks = 8;

// Argmax-word exchange between vocab-sharded ranks (one process per GPU).
// Every rank owns an exchange buffer in its own HBM, mapped into every
// other rank's address space (CUDA IPC, over NVLink):
//   words[2][nslots][world][B]  u64 argmax words, by (call parity, slot, writer)
//   flags[2][nslots][world]     u64 = the call's sequence number once written
// The last CTA of a launch that finishes slots [xslot0, xslot1) writes this
// rank's words into every rank's buffer, then the flags; the next cell kernel
// waits (bounded) for all ranks' flags of its slot and takes the max word.
struct Exchange {
  int world, rank;                         // world == 1: no exchange
  unsigned long long* peer[kMaxRanks];     // exchange buffer of rank j, as mapped here
  const unsigned long long* seq;           // sequence number of the current call (device)
  unsigned int* done;                      // per-slot count of finished CTAs (local)
  int nslots, B;
  unsigned long long timeout_ns;
  // Sharded s / gh phase: rank j raises sflags[(par * nslots + slot) * world + j]
  // (at u64 offset sflag_off of every buffer) once its slices of mid (byte
  // offset mid_off) and gh (gh_off) for that step are written.
  size_t sflag_off, mid_off, gh_off;
  unsigned int* sdone;  // per-slot finished-CTA counters of the s / gh phase (local)
};

__device__ __forceinline__ size_t xchg_word(const Exchange& x, int par, int slot, int writer, int b) {
  return (((size_t)par * x.nslots + slot) * x.world + writer) * x.B + b;
}
__device__ __forceinline__ size_t xchg_flag(const Exchange& x, int par, int slot, int writer) {
  return (size_t)2 * x.nslots * x.world * x.B + ((size_t)par * x.nslots + slot) * x.world + writer;
}

struct CellParams {
  int B, G, V;
  int src;                      // 0: token = ids[b * ids_ld + ids_col]; 1: token = argmax word
  const int64_t* ids;
  int ids_ld, ids_col;
  const unsigned long long* slots;  // word = slots[b * nslots + slot_idx]
  int nslots, slot_idx;
  int64_t* out;                 // if set: out[b * out_ld + out_col] = token
  int out_ld, out_col;
  int h_zero;                   // h = 0 and gh = b_hh (first prefix token)
  int write_h;
  int torch_cell;               // 1: the reference's PyTorch-branch cell, every op rounded, tanh (domino.py:423-430)
  const void* table;            // [V, 3G], row stride table_ld
  long long table_ld;
  const void* gh;               // [B, 3G]
  const void* b_hh;             // [3G] or null
  const void* h_in;             // [>=B, G]
  void* h_out;                  // [>=B, G]
  unsigned int* status;
  Exchange xchg;                // world > 1: the slot's word is the max over all ranks' words
  const unsigned long long* xbuf;  // this rank's exchange buffer
};

// Max over every rank's word for (slot, b), once all ranks have published it;
// 0 with DD_STATUS_TIMEOUT set if some rank has not within the time limit.
__device__ __forceinline__ unsigned long long gathered_word(const CellParams& p, int b, bool report) {
  const Exchange& x = p.xchg;
  const unsigned long long seq = *x.seq;
  const int par = (int)(seq & 1ull);
  unsigned long long best = 0ull;
  const uint64_t t0 = globaltimer_ns();
  for (int j = 0; j < x.world; ++j) {
    const unsigned long long* f = p.xbuf + xchg_flag(x, par, p.slot_idx, j);
    while (true) {
      unsigned long long v;
      asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(f) : "memory");
      if (v == seq) break;
      if (globaltimer_ns() - t0 > x.timeout_ns) {
        if (report) atomicOr(p.status, 1u /* DD_STATUS_TIMEOUT */);
        return best;
      }
      __nanosleep(64);
    }
    const unsigned long long w = __ldcv(p.xbuf + xchg_word(x, par, p.slot_idx, j, b));
    best = w > best ? w : best;
  }
  return best;
}

// Eight consecutive elements (16 bytes for 2-byte types, 32 for fp32; aligned).
template <typename T>
__device__ __forceinline__ void load8(const T* p, float (&f)[8]) {
  constexpr int kVecs = (int)sizeof(T) * 8 / 16;
  uint4 raw[kVecs];
#pragma unroll
  for (int v = 0; v < kVecs; ++v) raw[v] = reinterpret_cast<const uint4*>(p)[v];
  const T* e = reinterpret_cast<const T*>(raw);
#pragma unroll
  for (int i = 0; i < 8; ++i) f[i] = io<T>::to_f(e[i]);
}

// One thread's share of a GRU step: 8 state elements of one batch row
// (idx < B * G / 8).
template <typename T>
__device__ __forceinline__ void cell_apply(const CellParams& p, int idx) {
  const int per_row = p.G / 8;
  const int b = idx / per_row;
  const int g0 = (idx - b * per_row) * 8;

  long long tok;
  if (p.src == 0) {
    tok = p.ids[(size_t)b * p.ids_ld + p.ids_col];
  } else {
    const unsigned long long key =
        p.xchg.world > 1 ? gathered_word(p, b, g0 == 0) : p.slots[(size_t)b * p.nslots + p.slot_idx];
    if (key == 0ull) {
      if (g0 == 0) atomicOr(p.status, 4u /* DD_STATUS_NO_ARGMAX */);
      tok = 0;
    } else {
      tok = (long long)argmax_key_index(key);
    }
  }
  if (tok < 0 || tok >= p.V) {
    if (g0 == 0) atomicOr(p.status, 2u /* DD_STATUS_BAD_TOKEN */);
    tok = tok < 0 ? 0 : p.V - 1;
  }
  if (p.out && g0 == 0) p.out[(size_t)b * p.out_ld + p.out_col] = tok;
  if (!p.write_h) return;

  const int G = p.G;
  const T* gi = reinterpret_cast<const T*>(p.table) + (size_t)tok * p.table_ld;
  float ir[8], iz[8], in_[8], hr[8], hz[8], hn[8], h[8];
  load8<T>(gi + g0, ir);
  load8<T>(gi + G + g0, iz);
  load8<T>(gi + 2 * G + g0, in_);
  if (p.h_zero) {
    if (p.b_hh) {
      const T* bh = reinterpret_cast<const T*>(p.b_hh);
      load8<T>(bh + g0, hr);
      load8<T>(bh + G + g0, hz);
      load8<T>(bh + 2 * G + g0, hn);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) hr[i] = hz[i] = hn[i] = 0.0f;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) h[i] = 0.0f;
  } else {
    const T* ghr = reinterpret_cast<const T*>(p.gh) + (size_t)b * 3 * G;
    load8<T>(ghr + g0, hr);
    load8<T>(ghr + G + g0, hz);
    load8<T>(ghr + 2 * G + g0, hn);
    load8<T>(reinterpret_cast<const T*>(p.h_in) + (size_t)b * G + g0, h);
  }
  alignas(16) T outv[8];
  if (p.torch_cell) {
    // r = sigmoid(i_r + h_r); z = sigmoid(i_z + h_z); n = tanh(i_n + r * h_n);
    // h' = (1 - z) * n + z * h, each op's result in the state dtype
    auto rd = [](float x) { return io<T>::to_f(io<T>::from_f(x)); };
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float r = rd(sigmoidf_(rd(ir[i] + hr[i])));
      const float z = rd(sigmoidf_(rd(iz[i] + hz[i])));
      const float n = rd(tanhf(rd(in_[i] + rd(r * hn[i]))));
      outv[i] = io<T>::from_f(rd(rd(1.0f - z) * n) + rd(z * h[i]));
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float r = sigmoidf_(ir[i] + hr[i]);
      const float z = sigmoidf_(iz[i] + hz[i]);
      const float n = 2.0f * sigmoidf_(2.0f * (in_[i] + r * hn[i])) - 1.0f;
      outv[i] = io<T>::from_f((1.0f - z) * n + z * h[i]);
    }
  }
  constexpr int kVecs = (int)sizeof(T) * 8 / 16;
#pragma unroll
  for (int v = 0; v < kVecs; ++v)
    reinterpret_cast<uint4*>(reinterpret_cast<T*>(p.h_out) + (size_t)b * G + g0)[v] =
        reinterpret_cast<const uint4*>(outv)[v];
}

}  // namespace dd
