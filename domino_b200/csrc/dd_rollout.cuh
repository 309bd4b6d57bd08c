// dd_rollout.cuh -- the rollout of one draft block as ONE persistent kernel.
//
// The phased path launches one kernel per phase (s/gh projection, fc2 +
// argmax, GRU cell) and relies on programmatic dependent launch to overlap
// them.  Each launch still pays a ramp-up (first TMA round trip), a tail
// (last tile's epilogue and split-tile fix-up) and a launch gap; with the
// checkpoint-sized correction MLP (E ~ 1k) those fixed costs are about half
// of every step.  rollout_kernel runs every phase of the rollout in one
// cooperative launch (one CTA per SM, two pipelines per CTA, all resident):
//
//   * the TMA producer keeps two cursors over this CTA's units of all
//     phases: the weight cursor runs ahead across phase boundaries as far as
//     the ring allows (weights never depend on the recurrence), the
//     activation cursor waits until the phase before has completed on every
//     CTA (a grid-wide arrival counter per phase);
//   * the MMA warp and the epilogue warps walk the same phases in order;
//     after its last tile of a phase a CTA's epilogue warps add one arrival
//     to that phase's counter;
//   * GRU-cell phases run on the epilogue warps of every CTA (a slice of
//     batch x state each) once the phase before has completed everywhere.
//
// Every wait is bounded; the first CTA to time out raises a device-wide
// abort word and every other wait gives up on seeing it, so an error costs
// one time limit, not one per phase.
#pragma once

#include "dd_cell.cuh"

namespace dd {

enum RollPhaseType : int { RP_GEMV = 0, RP_CELL = 1 };
constexpr int kMaxRollPhases = 64;

struct RollPhase {
  int type;
  // RP_GEMV
  int nseg;
  GemvSeg seg[2];
  int a_map[2];  // RollMaps::a index of each segment's weight
  int b_map;     // RollMaps::b index of the activation operand
  int K, KC, N, n_valid, t;
  // RP_CELL (out_col < 0: the cell writes no token)
  int src, ids_col, slot_idx, out_col, h_zero, write_h, h_in, h_out;
};

struct RollMaps {
  CUtensorMap a[3];  // W_s, W_hh, fc2
  CUtensorMap b[3];  // h[0], h[1], mid
};

struct RollParams {
  GemvParams gp;  // fields shared by every phase's epilogue (shapes, pointers, scratch)
  CellParams cp;  // fields shared by every cell phase
  int nphases;
  RollPhase ph[kMaxRollPhases];
  void* hbuf[2];
  unsigned int* bar;         // [nphases] CTA arrivals per phase; zero at launch
  unsigned int* abort_word;  // device-wide abort; zero at launch
  int subs;                  // pipelines per CTA (1 or 2)
  int stages;
  uint32_t stage_bytes;      // 16 KB weight tile + n_max * 128 B activation slice
  int n_max;                 // TMEM columns per accumulator slot
  uint32_t tmem_cols;        // TMEM columns per pipeline
  uint32_t ab_fmt;           // 1 = bf16, 0 = fp16
};

__device__ __forceinline__ unsigned int ld_acquire_u32(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ long long phase_units(const RollPhase& P) {
  return (long long)(P.seg[0].tiles + (P.nseg > 1 ? P.seg[1].tiles : 0)) * P.KC;
}

// A walk over this CTA's units of every GEMV phase, in phase order.
struct UnitCursor {
  int ph;              // current phase (nphases when done)
  long long u, ue;     // unit and end of this CTA's range in the phase
  long long tile;
  int kc, KC;
  // the phase's fields the producer needs per unit, read once per phase
  int tiles0, row_tile0, row_tile1, a0, a1, b_map;
  uint32_t b_bytes;
};

__device__ __forceinline__ void cursor_seek(UnitCursor& cu, const RollParams& rp, int from, int c, int G) {
  for (int i = from; i < rp.nphases; ++i) {
    const RollPhase& P = rp.ph[i];
    if (P.type != RP_GEMV) continue;
    const long long U = phase_units(P);
    const long long b = unit_begin(c, U, G), e = unit_begin(c + 1, U, G);
    if (b < e) {
      cu.ph = i;
      cu.u = b;
      cu.ue = e;
      cu.KC = P.KC;
      cu.tile = b / P.KC;
      cu.kc = (int)(b - cu.tile * P.KC);
      cu.tiles0 = P.seg[0].tiles;
      cu.row_tile0 = P.seg[0].row_off / kTileM;
      cu.row_tile1 = P.seg[1].row_off / kTileM - P.seg[0].tiles;
      cu.a0 = P.a_map[0];
      cu.a1 = P.a_map[1];
      cu.b_map = P.b_map;
      cu.b_bytes = (uint32_t)P.N * 128u;
      return;
    }
  }
  cu.ph = rp.nphases;
}

__device__ __forceinline__ void cursor_next(UnitCursor& cu, const RollParams& rp, int c, int G) {
  ++cu.u;
  if (++cu.kc == cu.KC) {
    cu.kc = 0;
    ++cu.tile;
  }
  if (cu.u == cu.ue) cursor_seek(cu, rp, cu.ph + 1, c, G);
}

// Epilogue warps: wait until every CTA has arrived on `bar` (bounded; gives
// up at once when the device-wide abort word is set).  Collective over the
// 128 epilogue threads of one pipeline (named barrier `ebar`); true when the
// phase completed.
__device__ __forceinline__ bool grid_wait(const unsigned int* bar, unsigned int target, volatile unsigned int* gabort,
                                          volatile int* abort_flag, int ept, uint32_t ebar) {
  bool ok = true;
  if (ept == 0) {
    const uint64_t t0 = globaltimer_ns();
    while (ld_acquire_u32(bar) < target) {
      if (*gabort || *abort_flag) {
        ok = false;
        break;
      }
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        *gabort = 1u;
        *abort_flag = 1;
        ok = false;
        break;
      }
      __nanosleep(64);
    }
  }
  ok = named_bar_and(ebar, 128, ok);
  __threadfence();
  return ok;
}

// One CTA per SM holds rp.subs (1 or 2) independent pipelines of kThreads
// threads each: warp 0 TMA, warp 1 MMA, warps 2..5 epilogue, with their own
// ring, barriers and TMEM columns.  A cooperative launch admits only one
// TMEM-allocating CTA per SM, while streaming the weights at full HBM rate
// takes two pipelines per SM; pipeline s of CTA b acts as CTA
// s * gridDim.x + b of a grid of rp.subs * gridDim.x.
template <typename T>
__global__ void __launch_bounds__(2 * kThreads, 1)
    rollout_kernel(const __grid_constant__ RollMaps maps, const __grid_constant__ RollParams rp) {
  extern __shared__ uint8_t smem_raw[];
  const int sub = (int)threadIdx.x / kThreads;
  const int tid = (int)threadIdx.x - sub * kThreads;
  uint8_t* smem0 = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const size_t sub_bytes = (size_t)rp.stages * rp.stage_bytes + kSmemTail;
  uint8_t* ring = smem0 + (size_t)sub * sub_bytes;
  uint8_t* tail = ring + (size_t)rp.stages * rp.stage_bytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(tail);
  uint64_t* empty = full + kMaxStages;
  uint64_t* accf = empty + kMaxStages;
  uint64_t* acce = accf + 2;
  uint64_t* drain = acce + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  volatile int* fin_flag = abort_flag + 1;
  long long* issued = reinterpret_cast<long long*>(tail + 512);  // [0] weight loads, [2] activation loads
  long long* consumed = issued + 1;
  unsigned long long* red = reinterpret_cast<unsigned long long*>(tail + 1024);
  // pipeline 0's holder: the one TMEM allocation of the CTA
  uint32_t* tmem_holder0 = reinterpret_cast<uint32_t*>(smem0 + (size_t)rp.stages * rp.stage_bytes +
                                                       (size_t)(2 * kMaxStages + 5) * sizeof(uint64_t));
  volatile unsigned int* gabort = rp.abort_word;

  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int G = (int)gridDim.x * rp.subs;
  const int c = sub * (int)gridDim.x + (int)blockIdx.x;
  const uint32_t ebar = 1u + (uint32_t)sub;  // named barrier of this pipeline's epilogue warps

  if (tid == 0) {
    for (int s = 0; s < rp.stages; ++s) {
      mbar_init(&full[s], 2);  // weight tile + activation slice, each with its own expect_tx
      mbar_init(&empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&accf[s], 1);
      mbar_init(&acce[s], 128);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    *fin_flag = 0;
    issued[0] = 0;
    issued[2] = 0;
    *consumed = 0;
    fence_mbar_init();
  }
  if (sub == 0 && warp == 0 && lane == 0) {
    for (int i = 0; i < 3; ++i) {
      prefetch_tmap(&maps.a[i]);
      prefetch_tmap(&maps.b[i]);
    }
  }
  if (sub == 0 && warp == 1) {
    tmem_alloc(tmem_holder0, rp.tmem_cols * (uint32_t)rp.subs);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder0 + (uint32_t)sub * rp.tmem_cols;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------ TMA producer
      const uint64_t pol_w = policy_evict_first();
      const uint64_t pol_x = policy_evict_last();
      UnitCursor A, Bc;
      cursor_seek(A, rp, 0, c, G);
      cursor_seek(Bc, rp, 0, c, G);
      int sa = 0, sb = 0;
      uint32_t pa = 0;
      long long na = 0, nb = 0;
      int ready_upto = -1;       // phases [0, ready_upto] known complete on every CTA
      uint64_t stall_since = 0;  // read the timer only while nothing can be issued
      while (A.ph < rp.nphases || Bc.ph < rp.nphases) {
        // Activation load first: it is what the MMA is waiting for.
        bool b_blocked = false;
        if (Bc.ph < rp.nphases && nb < na) {
          const int need = Bc.ph - 1;  // the activations come from the phase before
          if (need > ready_upto && ld_acquire_u32(rp.bar + need) >= (unsigned int)G) {
            ready_upto = need;
            fence_proxy_async_global();  // generic stores of other CTAs -> this CTA's TMA reads
          }
          if (need <= ready_upto) {
            mbar_arrive_expect_tx(&full[sb], Bc.b_bytes);
            tma_load_2d(ring + (size_t)sb * rp.stage_bytes + kATileBytes, &maps.b[Bc.b_map], &full[sb],
                        Bc.kc * kChunkK, 0, pol_x);
            cursor_next(Bc, rp, c, G);
            ++nb;
            if (++sb == rp.stages) sb = 0;
            stall_since = 0;
            continue;
          }
          b_blocked = true;
        }
        if (A.ph < rp.nphases) {
          // With no activation load pending, park on the ring slot (the
          // hardware wakes us when it frees); otherwise only test it, so the
          // grid barrier is polled again.
          const bool got = b_blocked ? mbar_test_wait(&empty[sa], pa ^ 1u) : mbar_try_wait(&empty[sa], pa ^ 1u);
          if (got) {
            const bool s1 = A.tile >= A.tiles0;
            const long long w_tile = A.tile + (s1 ? A.row_tile1 : A.row_tile0);
            mbar_arrive_expect_tx(&full[sa], kATileBytes);
            tma_load_2d(ring + (size_t)sa * rp.stage_bytes, &maps.a[s1 ? A.a1 : A.a0], &full[sa], A.kc * kChunkK,
                        (int)(w_tile * kTileM), pol_w);
            cursor_next(A, rp, c, G);
            ++na;
            if (++sa == rp.stages) {
              sa = 0;
              pa ^= 1u;
            }
            stall_since = 0;
            continue;
          }
        }
        // The device-wide word lives in global memory: a read costs an L2 round
        // trip, so only a producer that is waiting on the grid anyway looks at
        // it; otherwise this pipeline's own roles raise the shared-memory flag.
        if (*abort_flag || (b_blocked && *gabort)) break;
        const uint64_t now = globaltimer_ns();
        if (stall_since == 0) {
          stall_since = now;
        } else if (now - stall_since > kWaitLimitNs) {
          *abort_flag = 1;
          *gabort = 1u;
          break;
        }
      }
      issued[0] = na;
      issued[2] = nb;
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------ MMA issuer
      long long it = 0;
      int stage = 0;
      uint32_t parity = 0;
      int acc_it = 0;
      bool ok = true;
      for (int i = 0; ok && i < rp.nphases; ++i) {
        const RollPhase& P = rp.ph[i];
        if (P.type != RP_GEMV) continue;
        const long long U = phase_units(P);
        const long long ub = unit_begin(c, U, G), ue = unit_begin(c + 1, U, G);
        const uint32_t idesc = idesc_f16((uint32_t)P.N, rp.ab_fmt);
        long long u = ub;
        while (ok && u < ue) {
          const long long tile = u / P.KC;
          const int kc0 = (int)(u - tile * P.KC);
          const long long left = ue - u;
          const int kc1 = (int)((P.KC - kc0) < left ? P.KC : kc0 + left);
          const int slot = acc_it & 1;
          const uint32_t use = (uint32_t)(acc_it >> 1);
          if (!mbar_wait_bounded(&acce[slot], (use & 1u) ^ 1u, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d = tmem_base + (uint32_t)(slot * rp.n_max);
          for (int kc = kc0; kc < kc1; ++kc, ++it) {
            if (!mbar_wait_bounded(&full[stage], parity, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t a_addr = smem_u32(ring + (size_t)stage * rp.stage_bytes);
            const uint64_t adesc = smem_desc_k_sw128(a_addr);
            const uint64_t bdesc = smem_desc_k_sw128(a_addr + kATileBytes);
#pragma unroll
            for (int k = 0; k < kChunkK / 16; ++k)
              mma_f16_ss(d, adesc + 2 * k, bdesc + 2 * k, idesc, (kc > kc0 || k > 0) ? 1u : 0u);
            mma_commit(&empty[stage]);
            if (++stage == rp.stages) {
              stage = 0;
              parity ^= 1u;
            }
          }
          if (!ok) break;
          mma_commit(&accf[slot]);
          ++acc_it;
          u += kc1 - kc0;
        }
      }
      if (!ok && !*abort_flag) *abort_flag = 1;
      if (*abort_flag) *gabort = 1u;
      *consumed = it;
    }
  } else {
    // ---------------------------------------- epilogue warps 2..5: tiles, cells, arrivals
    const int ept = tid - kEpiWarp0 * 32;
    // TMEM lane quarter: set by the warp's index within the CTA
    const int q = ((int)threadIdx.x >> 5) & 3;
    const int r = q * 32 + lane;
    int acc_it = 0;
    bool ok = true;
    for (int i = 0; ok && i < rp.nphases; ++i) {
      const RollPhase& P = rp.ph[i];
      if (P.type == RP_GEMV) {
        GemvParams p = rp.gp;
        p.nseg = P.nseg;
        p.seg[0] = P.seg[0];
        p.seg[1] = P.seg[1];
        p.K = P.K;
        p.KC = P.KC;
        p.N = P.N;
        p.n_off = 0;
        p.n_valid = P.n_valid;
        p.t = P.t;
        const long long U = phase_units(P);
        p.units = U;
        const int KC = P.KC;
        const long long ub = unit_begin(c, U, G), ue = unit_begin(c + 1, U, G);
        long long u = ub;
        while (u < ue) {
          const long long tile = u / KC;
          const int kc0 = (int)(u - tile * KC);
          const long long left = ue - u;
          const int kc1 = (int)((KC - kc0) < left ? KC : kc0 + left);
          const int slot = acc_it & 1;
          const uint32_t use = (uint32_t)(acc_it >> 1);
          const bool got = mbar_wait_bounded(&accf[slot], use & 1u, abort_flag);
          if (!named_bar_and(ebar, 128, got)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const bool s1 = tile >= p.seg[0].tiles;
          const GemvSeg& sg = p.seg[s1 ? 1 : 0];
          const int local_row = (int)((s1 ? tile - p.seg[0].tiles : tile) * kTileM) + r;
          const bool valid = local_row < sg.rows;
          const int row = sg.row_off + local_row;
          AccView a;
          a.taddr = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(slot * rp.n_max);
          a.nacc = 1;
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
          a.bar = ebar;
          a.xpose = nullptr;  // no X-row-major outputs in the rollout phases
          a.row0 = row - r;
          a.row_end = (long long)sg.row_off + sg.rows;
          bool finish = true;
          if (kc0 > 0 || kc1 < KC) {
            const int c_lo = cta_of_unit(tile * KC, U, G);
            const int c_hi = cta_of_unit(tile * KC + KC - 1, U, G);
            a.nseg = c_hi - c_lo + 1;
            a.myseg = c - c_lo;
            a.c_lo = c_lo;
            float* mine = p.partials + (size_t)partial_slot(c, tile, U, G, KC) * p.N * kTileM;
            for (int ch = 0; ch < p.N / 16; ++ch) {
              float v[16];
              acc_local(a, ch, v);
#pragma unroll
              for (int j = 0; j < 16; ++j) __stcg(mine + (size_t)(ch * 16 + j) * kTileM + r, v[j]);
            }
            __threadfence();
            named_bar_sync(ebar, 128);
            if (ept == 0) {
              const unsigned int old = atomicAdd(p.tile_counters + tile, 1u);
              const int lastseg = (old == (unsigned int)(a.nseg - 1)) ? 1 : 0;
              if (lastseg) {
                p.tile_counters[tile] = 0u;
                __threadfence();
              }
              *fin_flag = lastseg;
            }
            named_bar_sync(ebar, 128);
            finish = *fin_flag != 0;
            if (finish) {
              __threadfence();
              a.combine = true;
            }
          }
          if (finish) epilogue_tile<T, PH_ALL>(p, a, sg.kind, row, valid, q, lane, red, ept);
          tc_fence_before();
          mbar_arrive(&acce[slot]);
          ++acc_it;
          u += kc1 - kc0;
        }
        if (!ok) break;
      } else {
        // GRU cell over this CTA's slice of batch x state, once the phase
        // before (fc2 argmax, or the prefix gh) has completed everywhere.
        if (i > 0 && !grid_wait(rp.bar + (i - 1), (unsigned int)G, gabort, abort_flag, ept, ebar)) {
          ok = false;
          break;
        }
        CellParams cp = rp.cp;
        cp.src = P.src;
        cp.ids_col = P.ids_col;
        cp.slot_idx = P.slot_idx;
        cp.out_col = P.out_col;
        cp.out = P.out_col >= 0 ? rp.cp.out : nullptr;  // out_col < 0: this cell writes no token
        cp.h_zero = P.h_zero;
        cp.write_h = P.write_h;
        cp.h_in = rp.hbuf[P.h_in];
        cp.h_out = rp.hbuf[P.h_out];
        const int n = cp.B * (cp.G / 8);
        for (int idx = c * 128 + ept; idx < n; idx += G * 128) cell_apply<T>(cp, idx);
      }
      // This CTA is done with phase i.
      __threadfence();
      named_bar_sync(ebar, 128);
      if (ept == 0) atomicAdd(rp.bar + i, 1u);
    }
    if (!ok) {
      *abort_flag = 1;
      *gabort = 1u;
    }
  }

  __syncthreads();
  if (*abort_flag) {
    if (warp == 1 && lane == 0) {
      mma_commit(drain);
      wait_ns(drain, 0, 100ull * 1000 * 1000);
    }
    if (warp == 0 && lane == 0) {
      // Let every issued load land before the shared memory goes away.  A
      // stage whose activation load was never issued gets that arrival here
      // (no bytes), so its barrier completes once the weight tile has landed.
      for (long long it = *consumed; it < issued[0]; ++it) {
        uint64_t* f = &full[it % rp.stages];
        if (it >= issued[2]) mbar_arrive(f);
        wait_ns(f, (uint32_t)((it / rp.stages) & 1), 100ull * 1000 * 1000);
      }
    }
    if (tid == 0) atomicOr(rp.gp.status, 1u /* DD_STATUS_TIMEOUT */);
  }
  __syncthreads();
  tc_fence_after();
  if (sub == 0 && warp == 1) {
    __syncwarp();
    tmem_dealloc(*tmem_holder0, rp.tmem_cols * (uint32_t)rp.subs);
  }
}

}  // namespace dd
