// epoch_kernel.cuh -- the resident decode epoch as ONE persistent cooperative
// kernel for sm_100a (one CTA per SM).
//
// The kernel runs the whole epoch of the reference's device controller
// (controller/g4c_b4_resident_epoch.cpp:177-631) with no host involvement:
// validation, the one-shot KV import with its Adler-32 proof, generation
// continuity, then up to K full Qwen2 decoder steps
// (batched_decoder_step.py:277-417) each ending in a greedy argmax and the
// per-row EOS / max-step / slot / length bookkeeping.
//
// CTA layout: warps 0-7 are consumers (math, epilogues, control), warp 8 is
// the weight producer.  The producer streams every weight tile this CTA will
// consume, in consumption order, from HBM into a ring of shared-memory stages
// with 1-D bulk (TMA) copies completed on mbarriers.  Weights do not depend on
// activations, so it keeps prefetching across the grid barriers that separate
// phases; the consumers only wait for activations.
//
// Projection (GEMV) phases: y[4,N] = x[4,K] . W[N,K]^T.  W is cut into tiles of
// 16 rows x kc columns; the tiles of a phase are split into equal contiguous
// ranges over the CTAs ("stream-K"), so a row group may be split between two
// neighbouring CTAs: the upper part publishes fp32 partial sums, the lower
// part adds them in fixed order and runs the epilogue.  Inside a tile the 8
// consumer warps each take 64 columns and issue bf16 mma.sync m16n8k16 with W
// as the A operand and the 4 activation rows padded to n = 8 as B (the padding
// costs nothing: the phase is bandwidth bound).  A dot product may sum its k
// terms in any order, so each thread loads 16 contiguous weights per row with
// 128-bit shared loads and feeds them to four MMAs under one k permutation
// that the A and B fragments share.
//
// Every cross-CTA wait (grid barrier, split partial flag) and every mbarrier
// wait is bounded by a timeout; on expiry the kernel records status 207 and
// all CTAs leave, so a fault can never leave the GPU spinning.
#pragma once

#include <cfloat>
#include <climits>
#include <cstdint>

#include "epoch_types.h"
#include "ptx.cuh"

namespace cruise {

enum GemvKind : int32_t { kQKV = 0, kO = 1, kGU = 2, kDown = 3, kLM = 4 };
enum XMode : int32_t { kXNorm = 0, kXCopy = 1, kXGlobal = 2 };

struct Gemv {
  const bf16 *W;
  const bf16 *bias;      // kQKV only
  const bf16 *norm_w;    // kXNorm only
  const bf16 *xsrc;      // activation source, [4][xsrc_stride]
  int32_t N, K, kc, kind;
  int32_t xmode;
  int32_t xsrc_stride;
  int32_t embed_src;     // 1: the norm source is embed[token[b]] (layer 0)
};

__host__ __device__ inline int pick_kc(int K) {
  // largest power of two in 64..kMaxKc that divides K (K is a multiple of 64)
  for (int kc = kMaxKc; kc >= 64; kc >>= 1)
    if (K % kc == 0) return kc;
  return 64;
}

// Element offset of logical (n, k) inside a tiled matrix with K columns.
__host__ __device__ inline int64_t tiled_offset(int64_t n, int64_t k, int64_t K, int kc) {
  const int64_t rg = n / kRows, r = n % kRows;
  const int64_t kk = k / kc, kin = k % kc;
  const int64_t unit = (kin >> 3) ^ (r & 7);
  return ((rg * (K / kc) + kk) * kRows + r) * kc + unit * 8 + (kin & 7);
}

// The projection of a phase.  Under tensor parallelism the shapes are this
// rank's shard (O reads Hq attention columns, down I_pad columns of its rows);
// the residual stream h is whole on every rank.
__device__ __forceinline__ Gemv make_gemv(const EpochParams &p, int layer, int kind) {
  const ModelDims &m = p.m;
  Gemv g{};
  g.kind = kind;
  if (kind == kLM) {
    g.W = p.lm_head; g.N = m.V_pad; g.K = m.H;
    g.xmode = kXNorm; g.xsrc = p.h; g.xsrc_stride = m.H; g.norm_w = p.final_norm;
  } else {
    const LayerWeights &lw = p.layers[layer];
    switch (kind) {
      case kQKV:
        g.W = lw.qkv_w; g.bias = lw.qkv_b; g.N = m.Nqkv; g.K = m.H; g.xmode = kXNorm;
        g.xsrc = p.h; g.xsrc_stride = m.H; g.norm_w = lw.w_in; g.embed_src = layer == 0;
        break;
      case kO:
        g.W = lw.o_w; g.N = m.H; g.K = m.Kq; g.xmode = p.o_xglobal ? kXGlobal : kXCopy; g.xsrc = p.attn;
        g.xsrc_stride = m.Kq;   // attention output rows: Kq wide, columns >= Hq stay zero
        break;
      case kGU:
        g.W = lw.gu_w; g.N = 2 * m.I; g.K = m.H; g.xmode = kXNorm; g.xsrc = p.h;
        g.xsrc_stride = m.H; g.norm_w = lw.w_post;
        break;
      default:  // kDown
        g.W = lw.down_w; g.N = m.H; g.K = m.I_pad; g.xmode = p.down_xglobal ? kXGlobal : kXCopy;
        g.xsrc = p.act; g.xsrc_stride = m.I_pad;
        break;
    }
  }
  g.kc = pick_kc(g.K);
  return g;
}

struct TileRange {
  int64_t t0, t1;
  int32_t KT;      // tiles per row group
  int32_t ctas;    // CTAs that take part
};

// Equal contiguous tile ranges.  At most one CTA per row group of the phase
// takes part, so every range holds at least one full row group's worth of
// tiles and a row group is split between at most two neighbouring CTAs.
__device__ __forceinline__ TileRange tile_range(const Gemv &g, int cta, int grid) {
  TileRange r;
  r.KT = g.K / g.kc;
  const int64_t groups = g.N / kRows;
  const int64_t T = groups * r.KT;
  const int64_t ctas = groups < grid ? groups : grid;
  r.ctas = static_cast<int32_t>(ctas);
  if (cta >= ctas) {
    r.t0 = r.t1 = 0;
  } else {
    r.t0 = T * cta / ctas;
    r.t1 = T * (cta + 1) / ctas;
  }
  return r;
}

// The step program: per layer QKV, attention, O, gate/up, down; then lm_head
// and control.  Phase index within a step: 5*layer + {0..4}, 5L, 5L+1.
__device__ __forceinline__ int gemv_kind_of_phase(int ph, int L) {
  if (ph == 5 * L) return kLM;
  if (ph > 5 * L) return -1;  // control
  switch (ph % 5) {
    case 0: return kQKV;
    case 2: return kO;
    case 3: return kGU;
    case 4: return kDown;
    default: return -1;     // attention
  }
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---- shared memory map ------------------------------------------------------------
struct Smem {
  uint8_t *ring;           // stages x kStageBytes
  bf16 *xs;                // [4][xs_stride]  (attention and checksum scratch alias it)
  float *red;              // [kRedSlots][8 warps][64] row-group partial sums
  uint64_t *full;          // [kMaxStages]  weight stage landed
  uint64_t *empty;         // [kMaxStages]  weight stage consumed
  uint64_t *red_full;      // [kRedSlots]   partials written by the 8 consumer warps
  uint64_t *red_empty;     // [kRedSlots]   partials read by the epilogue warp
  uint64_t *phase_done;    // epilogue warp finished the current projection phase
  float *nrm;              // [8][4] norm partial sums, then [4] inverse rms at +32
  float *best_val;         // [8]
  int32_t *best_idx;       // [8]
  int32_t *best_bad;       // [8]
  int32_t *misc;           // [16] small broadcast values
  volatile int *prod_ctl;  // producer / epilogue control: -2 wait, >= s run step s, -1 stop
  volatile int *phase_started;  // sequence number of the projection phase the consumers began
  int64_t *row_pos;        // [4] row state of the current step (attention)
  int32_t *row_len;        // [4]
  int32_t *row_slot;       // [4]
  int32_t *row_act;        // [4]
  int32_t *bt;             // [4][kMaxBlocksPerRow] block table of the epoch
};

__host__ __device__ inline size_t smem_bytes(int stages, int xs_stride) {
  return static_cast<size_t>(stages) * kStageBytes + static_cast<size_t>(kBatch) * xs_stride * 2 +
         static_cast<size_t>(kRedSlots) * kConsumerWarps * 64 * 4 + 2 * kMaxStages * 8 +
         2 * kRedSlots * 8 + 8 + 40 * 4 + 24 * 4 + 16 * 4 + 16 + kBatch * 8 + 3 * kBatch * 4 +
         kBatch * kMaxBlocksPerRow * 4;
}

__device__ __forceinline__ Smem carve_smem(uint8_t *base, const EpochParams &p) {
  Smem s;
  uint8_t *ptr = base;
  s.ring = ptr;
  ptr += static_cast<size_t>(p.stages) * kStageBytes;
  s.xs = reinterpret_cast<bf16 *>(ptr);
  ptr += static_cast<size_t>(kBatch) * p.xs_stride * 2;
  s.red = reinterpret_cast<float *>(ptr);
  ptr += static_cast<size_t>(kRedSlots) * kConsumerWarps * 64 * 4;
  s.full = reinterpret_cast<uint64_t *>(ptr);
  ptr += kMaxStages * 8;
  s.empty = reinterpret_cast<uint64_t *>(ptr);
  ptr += kMaxStages * 8;
  s.red_full = reinterpret_cast<uint64_t *>(ptr);
  ptr += kRedSlots * 8;
  s.red_empty = reinterpret_cast<uint64_t *>(ptr);
  ptr += kRedSlots * 8;
  s.phase_done = reinterpret_cast<uint64_t *>(ptr);
  ptr += 8;
  s.nrm = reinterpret_cast<float *>(ptr);
  ptr += 40 * 4;
  s.best_val = reinterpret_cast<float *>(ptr);
  ptr += 8 * 4;
  s.best_idx = reinterpret_cast<int32_t *>(ptr);
  ptr += 8 * 4;
  s.best_bad = reinterpret_cast<int32_t *>(ptr);
  ptr += 8 * 4;
  s.misc = reinterpret_cast<int32_t *>(ptr);
  ptr += 16 * 4;
  s.prod_ctl = reinterpret_cast<volatile int *>(ptr);
  s.phase_started = reinterpret_cast<volatile int *>(ptr + 4);
  ptr += 16;
  s.row_pos = reinterpret_cast<int64_t *>(ptr);
  ptr += kBatch * 8;
  s.row_len = reinterpret_cast<int32_t *>(ptr);
  s.row_slot = s.row_len + kBatch;
  s.row_act = s.row_slot + kBatch;
  s.bt = s.row_act + kBatch;
  return s;
}

// Position in a ring of mbarrier-guarded slots.
struct RingCursor {
  uint32_t slot = 0;
  uint32_t parity = 0;
  __device__ __forceinline__ void advance(uint32_t n) {
    if (++slot == n) { slot = 0; parity ^= 1u; }
  }
};

// ---- cross-CTA helpers ---------------------------------------------------------------
__device__ __forceinline__ bool aborted(const EpochParams &p) {
  return *reinterpret_cast<volatile uint32_t *>(&p.sync->error) != 0;
}

__device__ __forceinline__ void raise_error(const EpochParams &p, uint32_t where) {
  if (atomicCAS(&p.sync->error, 0u, 1u) == 0u) p.sync->error_where = where;
}

// Grid barrier among the consumer warps of all CTAs.  `index` counts barriers
// from 1 within the launch.  Arrivals are spread over eight counters (CTA c
// adds to counter c % 8) so that they do not serialise on one L2 line; lanes
// 0-7 of warp 0 poll the eight counters in parallel with acquire loads and the
// CTA proceeds once every counter reached its target.
// Returns false when the launch is aborting.
__device__ bool grid_barrier(const EpochParams &p, const Smem &s, uint32_t index, uint32_t where) {
  named_sync(1, kConsumerThreads);
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    int ok = 1;
    if (lane == 0) {
      if (p.trace_cta != nullptr && index < kTraceMax)
        p.trace_cta[(static_cast<size_t>(index) * p.grid + blockIdx.x) * kTraceCtaWords + 3] = static_cast<uint32_t>(globaltimer());
      if (p.trace != nullptr && index < kTraceMax) {
        if (blockIdx.x == 0) p.trace[kTraceMax + index] = globaltimer();   // CTA 0 finished its share
        atomicMax(reinterpret_cast<unsigned long long *>(&p.trace[4 * kTraceMax + index]),
                  static_cast<unsigned long long>(globaltimer()));         // the last CTA to arrive
      }
      // every thread of the CTA wrote before the bar.sync above; the release
      // add makes those writes visible GPU-wide before the arrival is
      red_release_add_u32(&p.sync->barrier[blockIdx.x % kBarrierLanes][0], 1u);
    }
    const int grid = p.grid;
    const uint32_t members = lane < kBarrierLanes ? static_cast<uint32_t>((grid - lane + kBarrierLanes - 1) / kBarrierLanes) : 0u;
    const uint32_t target = index * members;
    const uint64_t deadline = globaltimer() + p.timeout_ns;
    for (uint32_t polls = 1;; ++polls) {
      // acquire: once a counter reached its target, the writes released
      // before those arrivals are visible to this lane
      const bool mine = lane >= kBarrierLanes ||
                        static_cast<int32_t>(ld_acquire_u32(&p.sync->barrier[lane][0]) - target) >= 0;
      if (__all_sync(0xffffffffu, mine)) break;
      if ((polls & 15) == 0) {
        int stop = 0;
        if (lane == 0) {
          if (aborted(p)) {
            stop = 1;
          } else if (globaltimer() > deadline) {
            raise_error(p, where);
            stop = 1;
          }
        }
        if (__shfl_sync(0xffffffffu, stop, 0)) { ok = 0; break; }
      }
    }
    __syncwarp();   // lanes 0-7's acquires order the CTA's reads after the bar.sync below
    if (lane == 0) {
      if (ok && aborted(p)) ok = 0;
      if (p.trace != nullptr && blockIdx.x == 0 && index < kTraceMax) p.trace[index] = globaltimer();
      if (p.trace_cta != nullptr && index < kTraceMax)
        p.trace_cta[(static_cast<size_t>(index) * p.grid + blockIdx.x) * kTraceCtaWords] = static_cast<uint32_t>(globaltimer());
      s.misc[0] = ok;
    }
  }
  named_sync(1, kConsumerThreads);
  return s.misc[0] != 0;
}

// Tensor parallelism: rank `src`'s partial in this rank's exchange block,
// once the word carries `tag` (the phase's sequence number).  A wait that runs
// out raises the epoch error and returns 0, so the kernel winds down.
__device__ __forceinline__ float tp_recv(const EpochParams &p, const uint64_t *word, uint32_t tag) {
  uint64_t v = ld_relaxed_sys_u64(word);
  if (static_cast<uint32_t>(v >> 32) != tag) {
    const uint64_t deadline = globaltimer() + p.timeout_ns;
    uint32_t polls = 0;
    while (static_cast<uint32_t>((v = ld_relaxed_sys_u64(word)) >> 32) != tag) {
      if ((++polls & 15) == 0) {
        if (aborted(p)) return 0.f;
        if (globaltimer() > deadline) { raise_error(p, 300); return 0.f; }
      }
    }
  }
  return __uint_as_float(static_cast<uint32_t>(v));
}

// QKV rows are q (heads of this rank) | k | v; every 16-row group lies inside
// one head (head_dim is a multiple of 16).  The KV head whose attention needs
// row group `rg`, and how many row groups one KV head's attention needs.
__device__ __forceinline__ int qkv_group_of(const ModelDims &m, int64_t rg) {
  const int64_t row = rg * kRows;
  const int groups = m.nq / m.nkv;
  if (row < m.Hq) return static_cast<int>(row / m.d) / groups;
  const int64_t kv = (row - m.Hq) / m.d;   // k heads, then v heads
  return static_cast<int>(kv < m.nkv ? kv : kv - m.nkv);
}

__device__ __forceinline__ uint32_t qkv_rows_per_group(const ModelDims &m) {
  return static_cast<uint32_t>((m.nq / m.nkv + 2) * (m.d / kRows));
}

// The fp32 value of a tagged partial-sum word once it carries `tag` (the
// phase's sequence number in the high half).  A wait that runs out raises the
// epoch error and returns 0, so the kernel winds down.
__device__ __forceinline__ float tagged_recv(const EpochParams &p, const uint64_t *word, uint32_t tag) {
  uint64_t v = ld_relaxed_gpu_u64(word);
  if (static_cast<uint32_t>(v >> 32) != tag) {
    const uint64_t deadline = globaltimer() + p.timeout_ns;
    uint32_t polls = 0;
    while (static_cast<uint32_t>((v = ld_relaxed_gpu_u64(word)) >> 32) != tag) {
      if ((++polls & 15) == 0) {
        if (aborted(p)) return 0.f;
        if (globaltimer() > deadline) { raise_error(p, 1001); return 0.f; }
      }
    }
  }
  return __uint_as_float(static_cast<uint32_t>(v));
}

// Slot of a position inside a row's valid range (32-bit: 0 <= t < C); -1 for
// an invalid block-table entry.  The attention's per-position lookup.
__device__ __forceinline__ int slot_in_row(const ModelDims &m, const int32_t *bt, int row, int t) {
  const int logical = t / m.bs;
  if (logical >= m.bpr) return -1;
  const int physical = bt[row * m.bpr + logical];
  if (physical < 0 || physical >= m.NB) return -1;
  return physical * m.bs + (t - logical * m.bs);
}

__device__ __forceinline__ int compute_slot(const ModelDims &m, const int32_t *bt, int row,
                                            int64_t position) {
  if (row < 0 || row >= kBatch || position < 0 || position >= m.C) return -1;
  const int logical = static_cast<int>(position / m.bs);
  const int offset = static_cast<int>(position % m.bs);
  if (logical >= m.bpr) return -1;
  const int physical = bt[row * m.bpr + logical];
  if (physical < 0 || physical >= m.NB) return -1;
  return physical * m.bs + offset;
}

// Waits for phase `parity` of `bar` with try_wait.  Gives up (false) when the
// launch aborts, when `*stop` reads -1, or after the launch's timeout.
__device__ __forceinline__ bool wait_bar(const EpochParams &p, uint64_t *bar, uint32_t parity,
                                         const volatile int *stop, uint32_t where) {
  if (mbar_try(bar, parity)) return true;
  const uint64_t deadline = globaltimer() + p.timeout_ns;
  for (uint32_t polls = 1;; ++polls) {
    if (mbar_try(bar, parity)) return true;
    if ((polls & 15) == 0) {
      if (aborted(p) || (stop != nullptr && *stop == -1)) return false;
      if (globaltimer() > deadline) {
        raise_error(p, where);
        return false;
      }
    }
  }
}

// Waits until the consumers release step `step` (true) or stop (false).
__device__ __forceinline__ bool wait_step(const EpochParams &p, const Smem &s, int step) {
  const uint64_t deadline = globaltimer() + p.timeout_ns;
  while (true) {
    const int ctl = *s.prod_ctl;   // -2 not yet released, -1 stop, s: run step s
    if (ctl == -1) return false;
    if (ctl >= step) return true;
    if (aborted(p) || globaltimer() > deadline) return false;
    __nanosleep(64);
  }
}

// ---- producer warp --------------------------------------------------------------------
// Streams the weight tiles of every projection phase of a step, in the order the
// consumers use them.  Waits for the consumers' go signal before each step.
// L2 run-ahead of the weight stream.  A second cursor walks the same
// (step, phase, tile) sequence as the bulk copies and keeps up to `l2_ahead`
// bytes of this CTA's future weight tiles in flight as L2 prefetches.  While
// the ring is full across a phase boundary (grid barrier, activation staging,
// attention) HBM keeps streaming into L2, and the copies into the ring that
// follow read L2 instead of waiting on DRAM.
struct L2RunAhead {
  int step = 0, ph = -1, steps = 0;
  int64_t t = 0, t1 = 0, tile_bytes = 0;
  const uint8_t *W = nullptr;
  uint64_t bytes = 0;   // issued so far

  uint64_t policy = 0;   // evict-last policy of the prefetched lines (l2_hints bit 1)

  __device__ void top_up(const EpochParams &p, uint64_t loaded) {
    const int L = p.m.L;
    const int phases = 5 * L + 2;
    while (step < steps && bytes < loaded + p.l2_ahead) {
      if (t >= t1) {   // next projection phase of the sequence
        if (++ph == phases) { ph = -1; ++step; continue; }
        const int kind = gemv_kind_of_phase(ph, L);
        if (kind < 0) continue;
        const Gemv g = make_gemv(p, ph / 5, kind);
        const TileRange tr = tile_range(g, blockIdx.x, p.grid);
        t = tr.t0;
        t1 = tr.t1;
        tile_bytes = static_cast<int64_t>(kRows) * g.kc * 2;
        W = reinterpret_cast<const uint8_t *>(g.W);
        continue;
      }
      const int64_t per = kStageBytes / tile_bytes;   // one ring stage's worth per prefetch
      const int64_t n = t1 - t < per ? t1 - t : per;
      if (p.l2_hints & 2u) {
        prefetch_l2_hint(W + t * tile_bytes, static_cast<uint32_t>(n * tile_bytes), policy);
      } else {
        prefetch_l2(W + t * tile_bytes, static_cast<uint32_t>(n * tile_bytes));
      }
      t += n;
      bytes += static_cast<uint64_t>(n * tile_bytes);
    }
  }
};

__device__ void producer_main(const EpochParams &p, const Smem &s) {
  const int lane = threadIdx.x & 31;
  const int L = p.m.L;
  const int phases = 5 * L + 2;
  RingCursor ring;
  uint32_t issued = 0;
  bool stop = false;
  L2RunAhead ahead;
  if (p.l2_hints & 2u) ahead.policy = l2_policy_evict_last();
  // weights are read once per step: their lines may leave L2 first once copied
  const uint64_t copy_policy = (p.l2_hints & 1u) ? l2_policy_evict_first() : 0;
  uint64_t loaded = 0;   // bytes of bulk copies issued into the ring
  for (int step = 0; step < kMaxSteps && !stop; ++step) {
    if (lane == 0) stop = !wait_step(p, s, step);
    stop = __shfl_sync(0xffffffffu, stop ? 1 : 0, 0) != 0;
    if (stop) break;
    if (step == 0 && lane == 0) ahead.steps = min(__ldcg(&p.work->max_steps), kMaxSteps);   // validated before step 0
    for (int ph = 0; ph < phases && !stop; ++ph) {
      const int kind = gemv_kind_of_phase(ph, L);
      if (kind < 0) continue;
      const Gemv g = make_gemv(p, ph / 5, kind);
      const TileRange tr = tile_range(g, blockIdx.x, p.grid);
      const int64_t tile_elems = static_cast<int64_t>(kRows) * g.kc;
      const int per_stage = kStageBytes / (kRows * g.kc * 2);
      for (int64_t t = tr.t0; t < tr.t1; t += per_stage) {
        const int n = static_cast<int>(tr.t1 - t < per_stage ? tr.t1 - t : per_stage);
        if (lane == 0) {
          if (p.l2_ahead != 0) ahead.top_up(p, loaded);
          stop = !wait_bar(p, &s.empty[ring.slot], ring.parity ^ 1u, s.prod_ctl, 900);
          if (!stop) {
            const uint32_t bytes = static_cast<uint32_t>(n * tile_elems * 2);
            loaded += bytes;
            mbar_arrive_expect_tx(&s.full[ring.slot], bytes);
            if (p.l2_hints & 1u) {
              bulk_g2s_hint(s.ring + static_cast<size_t>(ring.slot) * kStageBytes, g.W + t * tile_elems, bytes,
                            &s.full[ring.slot], copy_policy);
            } else {
              bulk_g2s(s.ring + static_cast<size_t>(ring.slot) * kStageBytes, g.W + t * tile_elems, bytes,
                       &s.full[ring.slot]);
            }
          }
        }
        stop = __shfl_sync(0xffffffffu, stop ? 1 : 0, 0) != 0;
        if (stop) break;
        ring.advance(p.stages);
        ++issued;
      }
    }
  }
  // Drain: every copy this warp issued must land before the CTA may exit.
  if (lane == 0) {
    const uint32_t first = issued > static_cast<uint32_t>(p.stages) ? issued - p.stages : 0u;
    for (uint32_t i = first; i < issued; ++i) {
      const uint64_t deadline = globaltimer() + p.timeout_ns;
      while (!mbar_try(&s.full[i % p.stages], (i / p.stages) & 1u)) {
        if (globaltimer() > deadline) break;
      }
    }
  }
  __syncwarp();
}

// ---- consumer: activation prologue ------------------------------------------------------
// Fills s.xs[4][K] with the projection input: RMSNorm of the residual stream
// (batched_decoder_step.py:224-229) or a plain copy (attention / SwiGLU output).
__device__ void load_x(const EpochParams &p, const Smem &s, const Gemv &g, uint32_t *mark) {
  const int tid = threadIdx.x;
  const int K = g.K;
  const int K8 = K / 8;
  if (g.xmode == kXCopy) {
    for (int i = tid; i < kBatch * K8; i += kConsumerThreads) {
      const int b = i / K8, k8 = i % K8;
      const uint4 v = __ldcg(reinterpret_cast<const uint4 *>(g.xsrc + static_cast<size_t>(b) * g.xsrc_stride) + k8);
      *reinterpret_cast<uint4 *>(s.xs + static_cast<size_t>(b) * p.xs_stride + k8 * 8) = v;
    }
    named_sync(1, kConsumerThreads);
    return;
  }
  // One pass over L2: each thread keeps its (at most 2 x 8) elements of every
  // row in registers (K <= 4096), reduces the fp32 sums of squares, then
  // normalises from registers.
  uint4 wv[2];   // norm weights, requested together with the activations
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int k8 = tid + j * kConsumerThreads;
    wv[j] = k8 < K8 ? __ldg(reinterpret_cast<const uint4 *>(g.norm_w) + k8) : make_uint4(0, 0, 0, 0);
  }
  const bf16 *rows[kBatch];
#pragma unroll
  for (int b = 0; b < kBatch; ++b) {
    rows[b] = g.embed_src ? p.embed + __ldcg(&p.work->token[b]) * static_cast<int64_t>(K)
                          : g.xsrc + static_cast<size_t>(b) * g.xsrc_stride;
  }
  uint4 v[2][kBatch];
  float ss[kBatch] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int k8 = tid + j * kConsumerThreads;
#pragma unroll
    for (int b = 0; b < kBatch; ++b) {
      v[j][b] = k8 < K8 ? __ldcg(reinterpret_cast<const uint4 *>(rows[b]) + k8) : make_uint4(0, 0, 0, 0);
      const __nv_bfloat162 *h2 = reinterpret_cast<const __nv_bfloat162 *>(&v[j][b]);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = __bfloat1622float2(h2[q]);
        ss[b] = __fadd_rn(ss[b], __fmul_rn(f.x, f.x));
        ss[b] = __fadd_rn(ss[b], __fmul_rn(f.y, f.y));
      }
    }
  }
  const int warp = tid >> 5, lane = tid & 31;
  if (mark != nullptr && tid == 0) mark[10] = static_cast<uint32_t>(globaltimer());   // loads returned
#pragma unroll
  for (int b = 0; b < kBatch; ++b) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ss[b] += __shfl_xor_sync(0xffffffffu, ss[b], off);
  }
  if (lane == 0) {
#pragma unroll
    for (int b = 0; b < kBatch; ++b) s.nrm[warp * 4 + b] = ss[b];
  }
  named_sync(1, kConsumerThreads);
  if (mark != nullptr && tid == 0) mark[11] = static_cast<uint32_t>(globaltimer());   // sums shared
  // every warp sums the 8 warp partials in the same order, lane b computing
  // row b's inverse RMS, and broadcasts the four values by shuffles (no
  // second barrier; one IEEE divide / square root / divide chain per lane)
  float mine = 0.f;
  if (lane < kBatch) {
    float total = 0.f;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) total += s.nrm[w * 4 + lane];
    // mean = sum / K; rsqrt = 1 / sqrt(mean + eps), each IEEE-rounded as on the CPU
    const float var = __fdiv_rn(total, static_cast<float>(K));
    mine = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, p.m.eps)));
  }
  float rinv[kBatch];
#pragma unroll
  for (int b = 0; b < kBatch; ++b) rinv[b] = __shfl_sync(0xffffffffu, mine, b);
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int k8 = tid + j * kConsumerThreads;
    if (k8 >= K8) continue;
    const __nv_bfloat162 *w2 = reinterpret_cast<const __nv_bfloat162 *>(&wv[j]);
#pragma unroll
    for (int b = 0; b < kBatch; ++b) {
      const float r = rinv[b];
      const __nv_bfloat162 *h2 = reinterpret_cast<const __nv_bfloat162 *>(&v[j][b]);
      uint4 o;
      __nv_bfloat162 *o2 = reinterpret_cast<__nv_bfloat162 *>(&o);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 hf = __bfloat1622float2(h2[q]);
        const float2 wf = __bfloat1622float2(w2[q]);
        const float nx = rbf(__fmul_rn(hf.x, r));   // (h * rsqrt).to(bf16)
        const float ny = rbf(__fmul_rn(hf.y, r));
        o2[q] = __floats2bfloat162_rn(__fmul_rn(nx, wf.x), __fmul_rn(ny, wf.y));  // * weight
      }
      *reinterpret_cast<uint4 *>(s.xs + static_cast<size_t>(b) * p.xs_stride + k8 * 8) = o;
    }
  }
  named_sync(1, kConsumerThreads);
}

// Flushes one warp's 16 x 4 partial sums of a finished row-group segment to
// the epilogue warp through the reduction ring.
__device__ __forceinline__ void flush_segment(const EpochParams &p, const Smem &s, RingCursor &red, int warp,
                                              int lane, float (&acc)[4], float (&acc2)[4]) {
  const int gi = lane >> 2, ci = lane & 3;
  wait_bar(p, &s.red_empty[red.slot], red.parity ^ 1u, nullptr, 1002);
  if (ci < 2) {
    float *r = s.red + (static_cast<size_t>(red.slot) * kConsumerWarps + warp) * 64;
    r[gi * 4 + 2 * ci] = acc[0] + acc2[0];
    r[gi * 4 + 2 * ci + 1] = acc[1] + acc2[1];
    r[(gi + 8) * 4 + 2 * ci] = acc[2] + acc2[2];
    r[(gi + 8) * 4 + 2 * ci + 1] = acc[3] + acc2[3];
  }
  __syncwarp();
  if (lane == 0) mbar_arrive(&s.red_full[red.slot]);
  red.advance(kRedSlots);
  acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
  acc2[0] = acc2[1] = acc2[2] = acc2[3] = 0.f;
}

// Tile loop for kc = 512 (every 7B-shaped projection): warp w owns the 64-k
// slice w of every tile and a stage holds two tiles.  Per stage all shared
// loads of both tiles (8 A fragments, 4 activation fragments) are issued
// before the 8 MMAs, so a stage costs one shared-memory latency; addresses are
// precomputed per warp.  kXGlobal keeps the activation fragments of the next
// four tiles in flight from L2, as in the general loop.
__device__ void gemv_tiles_k512(const EpochParams &p, const Smem &s, const Gemv &g, const TileRange &tr,
                                RingCursor &ring, RingCursor &red) {
  constexpr int kc = 64 * kConsumerWarps;
  constexpr uint32_t row_bytes = kc * 2, tile_bytes = row_bytes * kRows;
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int gi = lane >> 2, ci = lane & 3;
  const uint32_t sw = static_cast<uint32_t>(gi & 7);
  const uint32_t off_lo0 = gi * row_bytes + ((static_cast<uint32_t>(warp * 8 + 2 * ci) ^ sw) << 4);
  const uint32_t off_lo1 = gi * row_bytes + ((static_cast<uint32_t>(warp * 8 + 2 * ci + 1) ^ sw) << 4);
  const uint32_t off_hi0 = off_lo0 + 8 * row_bytes, off_hi1 = off_lo1 + 8 * row_bytes;
  const bool xg = g.xmode == kXGlobal;
  const bool xlane = gi < kBatch;
  // staged activations: row gi, k = kk * kc + warp * 64 + 16 ci (+8)
  const bf16 *xs_row = s.xs + static_cast<size_t>(xlane ? gi : 0) * p.xs_stride + warp * 64 + 16 * ci;
  const bf16 *xg_base = g.xsrc + static_cast<size_t>(xlane ? gi : 0) * g.xsrc_stride + warp * 64 + 16 * ci;
  const int KT = tr.KT;
  const int count = static_cast<int>(tr.t1 - tr.t0);
  int kk = static_cast<int>(tr.t0 % KT);   // k tile of the next tile
  int kq = kk;                              // k tile of the next L2 prefetch (kXGlobal)
  auto xg_load = [&](int i, uint4 &lo, uint4 &hi) {
    if (xg && xlane && i < count) {
      const uint4 *src = reinterpret_cast<const uint4 *>(xg_base + static_cast<int64_t>(kq) * kc);
      lo = __ldcg(src);
      hi = __ldcg(src + 1);
    } else {
      lo = make_uint4(0, 0, 0, 0);
      hi = make_uint4(0, 0, 0, 0);
    }
    kq = kq + 1 == KT ? 0 : kq + 1;
  };
  uint4 x00, x01, x10, x11, x20, x21, x30, x31;
  xg_load(0, x00, x01);
  xg_load(1, x10, x11);
  xg_load(2, x20, x21);
  xg_load(3, x30, x31);
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  float acc2[4] = {0.f, 0.f, 0.f, 0.f};
  // loop-invariant state in registers
  const uint8_t *const ring_base = s.ring;
  uint64_t *const full = s.full;
  uint64_t *const empty = s.empty;
  const int stages = p.stages;
  for (int i = 0; i < count; i += 2) {
    const bool two = i + 1 < count;
    const bool landed = wait_bar(p, full + ring.slot, ring.parity, nullptr, 1000);
    const uint8_t *t0 = ring_base + static_cast<size_t>(ring.slot) * kStageBytes;
    const uint8_t *t1 = t0 + tile_bytes;
    const int kk1 = kk + 1 == KT ? 0 : kk + 1;
    // all shared loads of the stage first
    const uint4 a0lo0 = lds128(t0 + off_lo0), a0lo1 = lds128(t0 + off_lo1);
    const uint4 a0hi0 = lds128(t0 + off_hi0), a0hi1 = lds128(t0 + off_hi1);
    uint4 a1lo0 = make_uint4(0, 0, 0, 0), a1lo1 = a1lo0, a1hi0 = a1lo0, a1hi1 = a1lo0;
    if (two) {
      a1lo0 = lds128(t1 + off_lo0);
      a1lo1 = lds128(t1 + off_lo1);
      a1hi0 = lds128(t1 + off_hi0);
      a1hi1 = lds128(t1 + off_hi1);
    }
    uint4 xa0 = x00, xa1 = x01, xb0 = x10, xb1 = x11;
    if (!xg && xlane) {
      xa0 = lds128(xs_row + kk * kc);
      xa1 = lds128(xs_row + kk * kc + 8);
      if (two) {
        xb0 = lds128(xs_row + kk1 * kc);
        xb1 = lds128(xs_row + kk1 * kc + 8);
      }
    }
    // L2 prefetch of the activation fragments four tiles ahead (kXGlobal)
    x00 = x20; x01 = x21; x10 = x30; x11 = x31;
    xg_load(i + 4, x20, x21);
    xg_load(i + 5, x30, x31);
    // tile 0
    mma_bf16_16816(acc, a0lo0.x, a0hi0.x, a0lo0.y, a0hi0.y, xa0.x, xa0.y);
    mma_bf16_16816(acc2, a0lo0.z, a0hi0.z, a0lo0.w, a0hi0.w, xa0.z, xa0.w);
    mma_bf16_16816(acc, a0lo1.x, a0hi1.x, a0lo1.y, a0hi1.y, xa1.x, xa1.y);
    mma_bf16_16816(acc2, a0lo1.z, a0hi1.z, a0lo1.w, a0hi1.w, xa1.z, xa1.w);
    if (kk == KT - 1 || i == count - 1) flush_segment(p, s, red, warp, lane, acc, acc2);
    if (two) {
      mma_bf16_16816(acc, a1lo0.x, a1hi0.x, a1lo0.y, a1hi0.y, xb0.x, xb0.y);
      mma_bf16_16816(acc2, a1lo0.z, a1hi0.z, a1lo0.w, a1hi0.w, xb0.z, xb0.w);
      mma_bf16_16816(acc, a1lo1.x, a1hi1.x, a1lo1.y, a1hi1.y, xb1.x, xb1.y);
      mma_bf16_16816(acc2, a1lo1.z, a1hi1.z, a1lo1.w, a1hi1.w, xb1.z, xb1.w);
      if (kk1 == KT - 1 || i + 1 == count - 1) flush_segment(p, s, red, warp, lane, acc, acc2);
    }
    kk = kk1 + 1 == KT ? 0 : kk1 + 1;
    if (!two) kk = kk1;
    __syncwarp();
    if (lane == 0 && landed) mbar_arrive(empty + ring.slot);
    ring.advance(stages);
  }
}

// General tile loop (any kc): each warp takes the 64-k slices warp, warp + 8,
// ... of every tile.
__device__ void gemv_tiles_general(const EpochParams &p, const Smem &s, const Gemv &g, const TileRange &tr,
                                   RingCursor &ring, RingCursor &red) {
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int gi = lane >> 2, ci = lane & 3;
  const bool xg = g.xmode == kXGlobal;
  const int kc = g.kc;
  const int ksteps = kc / 64;
  const uint32_t row_bytes = static_cast<uint32_t>(kc) * 2u;
  const uint32_t tile_bytes = row_bytes * kRows;
  const int per_stage = kStageBytes / static_cast<int>(tile_bytes);
  const uint32_t sw = static_cast<uint32_t>(gi & 7);   // row swizzle of rows gi and gi + 8
  // two accumulator sets halve the dependent MMA chain of a tile
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  float acc2[4] = {0.f, 0.f, 0.f, 0.f};
  // kXGlobal (one 64-wide k-step per warp and tile): each thread with gi < 4
  // keeps the activation fragments of the next four tiles in flight from L2.
  const bf16 *xg_base = g.xsrc + static_cast<size_t>(gi) * g.xsrc_stride + warp * 64 + 16 * ci;
  const bool xg_lane = xg && gi < kBatch;
  auto xg_load = [&](int64_t tt, int tkk, uint4 &lo, uint4 &hi) {
    if (xg_lane && tt < tr.t1) {
      const uint4 *src = reinterpret_cast<const uint4 *>(xg_base + static_cast<int64_t>(tkk) * kc);
      lo = __ldcg(src);
      hi = __ldcg(src + 1);
    } else {
      lo = make_uint4(0, 0, 0, 0);
      hi = make_uint4(0, 0, 0, 0);
    }
  };
  auto next_kk = [&](int v) { return v + 1 == tr.KT ? 0 : v + 1; };
  int kk = static_cast<int>(tr.t0 % tr.KT);
  int kq = kk;   // k-tile of the next prefetch
  uint4 x00, x01, x10, x11, x20, x21, x30, x31;
  xg_load(tr.t0, kq, x00, x01); kq = next_kk(kq);
  xg_load(tr.t0 + 1, kq, x10, x11); kq = next_kk(kq);
  xg_load(tr.t0 + 2, kq, x20, x21); kq = next_kk(kq);
  for (int64_t t = tr.t0; t < tr.t1;) {
    const int n = static_cast<int>(tr.t1 - t < per_stage ? tr.t1 - t : per_stage);
    // Bounded wait.  On abort or timeout the phase still runs to its end (on
    // garbage) so that every barrier below is matched; the grid barrier that
    // ends the phase then stops the launch uniformly.
    const bool landed = wait_bar(p, &s.full[ring.slot], ring.parity, nullptr, 1000);
    const uint8_t *stage = s.ring + static_cast<size_t>(ring.slot) * kStageBytes;
    for (int j = 0; j < n; ++j, ++t) {
      xg_load(t + 3, kq, x30, x31);
      kq = next_kk(kq);
      const uint8_t *tile = stage + j * tile_bytes;
      for (int ks = warp; ks < ksteps; ks += kConsumerWarps) {
        const uint32_t u0 = (static_cast<uint32_t>(ks * 8 + 2 * ci) ^ sw) * 16u;
        const uint32_t u1 = (static_cast<uint32_t>(ks * 8 + 2 * ci + 1) ^ sw) * 16u;
        const uint8_t *rlo = tile + gi * row_bytes;
        const uint8_t *rhi = rlo + 8 * row_bytes;
        const uint4 a_lo0 = lds128(rlo + u0);
        const uint4 a_lo1 = lds128(rlo + u1);
        const uint4 a_hi0 = lds128(rhi + u0);
        const uint4 a_hi1 = lds128(rhi + u1);
        uint4 x0 = x00, x1 = x01;
        if (!xg && gi < kBatch) {
          const bf16 *xrow = s.xs + static_cast<size_t>(gi) * p.xs_stride + kk * kc + ks * 64 + 16 * ci;
          x0 = lds128(xrow);
          x1 = lds128(xrow + 8);
        }
        // MMA j uses physical k = 16ci + 4j .. 4j+3 of this 64-wide slice, for both
        // weight rows (gi, gi+8) and the activation column gi.
        mma_bf16_16816(acc, a_lo0.x, a_hi0.x, a_lo0.y, a_hi0.y, x0.x, x0.y);
        mma_bf16_16816(acc2, a_lo0.z, a_hi0.z, a_lo0.w, a_hi0.w, x0.z, x0.w);
        mma_bf16_16816(acc, a_lo1.x, a_hi1.x, a_lo1.y, a_hi1.y, x1.x, x1.y);
        mma_bf16_16816(acc2, a_lo1.z, a_hi1.z, a_lo1.w, a_hi1.w, x1.z, x1.w);
      }
      x00 = x10; x01 = x11; x10 = x20; x11 = x21; x20 = x30; x21 = x31;
      if (kk == tr.KT - 1 || t == tr.t1 - 1) {
        // segment end: this warp's 16 x 4 partial sums go to the epilogue warp
        wait_bar(p, &s.red_empty[red.slot], red.parity ^ 1u, nullptr, 1002);
        if (ci < 2) {
          float *r = s.red + (static_cast<size_t>(red.slot) * kConsumerWarps + warp) * 64;
          r[gi * 4 + 2 * ci] = acc[0] + acc2[0];
          r[gi * 4 + 2 * ci + 1] = acc[1] + acc2[1];
          r[(gi + 8) * 4 + 2 * ci] = acc[2] + acc2[2];
          r[(gi + 8) * 4 + 2 * ci + 1] = acc[3] + acc2[3];
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&s.red_full[red.slot]);
        red.advance(kRedSlots);
        acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
        acc2[0] = acc2[1] = acc2[2] = acc2[3] = 0.f;
      }
      kk = next_kk(kk);
    }
    __syncwarp();
    if (lane == 0 && landed) mbar_arrive(&s.empty[ring.slot]);
    ring.advance(p.stages);
  }
}

// ---- consumer warps: one projection phase ---------------------------------------------------
// Streams this CTA's tiles through the MMA and hands every finished row-group
// segment (fp32 partials of 16 rows x 4 batch rows per warp) to the epilogue
// warp through the reduction ring; no CTA-wide synchronisation in the stream.
__device__ void gemv_consume(const EpochParams &p, const Smem &s, const Gemv &g, RingCursor &ring,
                             RingCursor &red, uint32_t trace_slot) {
  const int tid = threadIdx.x;
  const TileRange tr = tile_range(g, blockIdx.x, p.grid);
  if (g.embed_src) {
    // layer 0: every CTA materialises its slice of the residual stream h = E[token]
    const int K8 = g.K / 8;
    const int lo = static_cast<int>(static_cast<int64_t>(K8) * blockIdx.x / p.grid);
    const int hi = static_cast<int>(static_cast<int64_t>(K8) * (blockIdx.x + 1) / p.grid);
    for (int i = tid; i < kBatch * (hi - lo); i += kConsumerThreads) {
      const int b = i / (hi - lo), k8 = lo + i % (hi - lo);
      const int64_t tok = __ldcg(&p.work->token[b]);
      const uint4 v = __ldcg(reinterpret_cast<const uint4 *>(p.embed + tok * g.K) + k8);
      *reinterpret_cast<uint4 *>(p.h + static_cast<size_t>(b) * p.m.H + k8 * 8) = v;
    }
  }
  if (tr.t0 >= tr.t1) return;
  const bool xg = g.xmode == kXGlobal;
  if (!xg)
    load_x(p, s, g,
           p.trace_cta != nullptr && trace_slot < kTraceMax
               ? p.trace_cta + (static_cast<size_t>(trace_slot) * p.grid + blockIdx.x) * kTraceCtaWords
               : nullptr);
  if (p.trace != nullptr && blockIdx.x == 0 && tid == 0 && trace_slot < kTraceMax)
    p.trace[2 * kTraceMax + trace_slot] = globaltimer();   // activations staged
  if (p.trace_cta != nullptr && tid == 0 && trace_slot < kTraceMax)
    p.trace_cta[(static_cast<size_t>(trace_slot) * p.grid + blockIdx.x) * kTraceCtaWords + 1] = static_cast<uint32_t>(globaltimer());
  if (g.kc == 64 * kConsumerWarps && kStageBytes / (kRows * g.kc * 2) == 2) {
    gemv_tiles_k512(p, s, g, tr, ring, red);
  } else {
    gemv_tiles_general(p, s, g, tr, ring, red);
  }
  if (p.trace != nullptr && blockIdx.x == 0 && tid == 0 && trace_slot < kTraceMax)
    p.trace[3 * kTraceMax + trace_slot] = globaltimer();   // last tile consumed by warp 0
  if (p.trace_cta != nullptr && tid == 0 && trace_slot < kTraceMax)
    p.trace_cta[(static_cast<size_t>(trace_slot) * p.grid + blockIdx.x) * kTraceCtaWords + 2] = static_cast<uint32_t>(globaltimer());
  if (p.trace_cta != nullptr && (tid & 31) == 0 && trace_slot < kTraceMax)   // the last consumer warp done
    atomicMax(&p.trace_cta[(static_cast<size_t>(trace_slot) * p.grid + blockIdx.x) * kTraceCtaWords + 9],
              static_cast<uint32_t>(globaltimer()));
}

// ---- epilogue warp: one projection phase --------------------------------------------------------
// Lane l owns rows (l/4, l/4 + 8) of the row group and batch row l%4.  For each
// segment it sums the 8 warps' partials in fixed order, then either publishes
// them (the segment's row group started on the previous CTA), or adds the next
// CTA's published part (the row group continues there) and runs the epilogue.
__device__ void gemv_finish(const EpochParams &p, const Smem &s, const Gemv &g, RingCursor &red,
                            uint32_t seq, int step, uint32_t trace_slot) {
  const int lane = threadIdx.x & 31;
  const ModelDims &m = p.m;
  const TileRange tr = tile_range(g, blockIdx.x, p.grid);
  // per-CTA trace of the epilogue warp: [4] started, [5] ns waited for the
  // stream-K partner, [6] last segment done, [7] outputs fenced
  uint32_t *const mark = p.trace_cta != nullptr && trace_slot < kTraceMax
                             ? p.trace_cta + (static_cast<size_t>(trace_slot) * p.grid + blockIdx.x) * kTraceCtaWords
                             : nullptr;
  uint64_t partner_ns = 0;
  if (mark != nullptr && lane == 0) mark[4] = static_cast<uint32_t>(globaltimer());
  float best = -INFINITY;
  int32_t best_i = INT_MAX, bad = 0;

  int64_t seg_start = tr.t0;
  int64_t rg = tr.t0 / tr.KT;
  int kk = static_cast<int>(tr.t0 % tr.KT);
  // Operands of the epilogue that do not depend on this phase's sums (residual
  // rows, biases) are loaded up front for the first two row groups this CTA
  // finishes; the small projections have at most two.
  const int b_lane = lane & 3;
  float pa0 = 0.f, pa1 = 0.f, pb0 = 0.f, pb1 = 0.f;
  int64_t pa_rg = -1, pb_rg = -1;
  const bool tp_partial = p.tp_size > 1 && (g.kind == kO || g.kind == kDown);
  // lane r < tp_size holds rank r's exchange block (shuffled to every lane per send)
  TpExchange *const peer_mine = tp_partial && lane < p.tp_size ? p.tp_peer[lane] : nullptr;
  if (g.kind == kQKV || g.kind == kO || g.kind == kDown) {
    const int64_t first_head = tr.t0 % tr.KT == 0 ? tr.t0 / tr.KT : tr.t0 / tr.KT + 1;
    auto fetch = [&](int64_t r, float &v0, float &v1) {
      const int64_t n0 = r * kRows + (lane >> 2), n1 = n0 + 8;
      if (g.kind == kQKV) {
        v0 = bf(g.bias[n0]);
        v1 = bf(g.bias[n1]);
      } else {
        v0 = bf(__ldcg(p.h + static_cast<size_t>(b_lane) * m.H + n0));
        v1 = bf(__ldcg(p.h + static_cast<size_t>(b_lane) * m.H + n1));
      }
    };
    if (first_head * tr.KT < tr.t1) { pa_rg = first_head; fetch(pa_rg, pa0, pa1); }
    if ((first_head + 1) * tr.KT < tr.t1) { pb_rg = first_head + 1; fetch(pb_rg, pb0, pb1); }
  }
  for (int64_t t = tr.t0; t < tr.t1; ++t) {
    const bool group_end = kk == tr.KT - 1;
    if (group_end || t == tr.t1 - 1) {
      const bool head_seg = (seg_start % tr.KT) == 0;
      float part0 = 0.f, part1 = 0.f;
      if (head_seg && !group_end) {
        // finisher: the next CTA publishes the rest of this row group early in
        // its range as tagged words; each lane takes its two once their tag
        // is this phase's (an aligned 64-bit access is single-copy atomic)
        const uint64_t wait0 = globaltimer();
        part0 = tagged_recv(p, p.partials + static_cast<size_t>(blockIdx.x + 1) * 64 + lane, seq);
        part1 = tagged_recv(p, p.partials + static_cast<size_t>(blockIdx.x + 1) * 64 + lane + 32, seq);
        if (lane == 0) partner_ns += globaltimer() - wait0;
      }
      wait_bar(p, &s.red_full[red.slot], red.parity, s.prod_ctl, 1003);
      if (mark != nullptr && lane == 0) mark[8] = static_cast<uint32_t>(globaltimer());
      const float *r = s.red + static_cast<size_t>(red.slot) * kConsumerWarps * 64;
      float v0 = 0.f, v1 = 0.f;
#pragma unroll
      for (int w = 0; w < kConsumerWarps; ++w) {
        v0 += r[w * 64 + lane];
        v1 += r[w * 64 + lane + 32];
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.red_empty[red.slot]);
      red.advance(kRedSlots);
      const bool head = head_seg;   // this CTA holds the group's first tile
      seg_start = t + 1;
      if (!head) {
        // publish this CTA's part of the row group to the finisher (CTA - 1)
        const uint64_t tag = static_cast<uint64_t>(seq) << 32;
        st_relaxed_gpu_u64(p.partials + static_cast<size_t>(blockIdx.x) * 64 + lane, tag | __float_as_uint(v0));
        st_relaxed_gpu_u64(p.partials + static_cast<size_t>(blockIdx.x) * 64 + lane + 32, tag | __float_as_uint(v1));
      } else {
        if (!group_end) {   // the rest of the row group came from CTA + 1
          v0 += part0;
          v1 += part1;
        }
        const int b = b_lane;
        const int64_t n0 = rg * kRows + (lane >> 2), n1 = n0 + 8;
        float e0, e1;   // bias (QKV) or residual (O, down) of rows n0, n1
        if (rg == pa_rg) {
          e0 = pa0;
          e1 = pa1;
        } else if (rg == pb_rg) {
          e0 = pb0;
          e1 = pb1;
        } else if (g.kind == kQKV) {
          e0 = bf(g.bias[n0]);
          e1 = bf(g.bias[n1]);
        } else if (g.kind == kO || g.kind == kDown) {
          e0 = bf(__ldcg(p.h + static_cast<size_t>(b) * m.H + n0));
          e1 = bf(__ldcg(p.h + static_cast<size_t>(b) * m.H + n1));
        } else {
          e0 = e1 = 0.f;
        }
        if (g.kind == kQKV) {
          // F.linear(x, W, b) on bf16: fp32 sum plus fp32 bias, one rounding (:305-313)
          p.qkv[static_cast<size_t>(b) * m.Nqkv + n0] = tobf(__fadd_rn(v0, e0));
          p.qkv[static_cast<size_t>(b) * m.Nqkv + n1] = tobf(__fadd_rn(v1, e1));
          // the row group is complete: count it for its KV head's attention
          // (the warp's stores are ordered before lane 0's release add)
          __syncwarp();
          if (lane == 0) red_release_add_u32(&p.sync->qkv_done[qkv_group_of(m, rg)][0], 1u);
        } else if (tp_partial) {
          // Row-parallel output under tensor parallelism: every rank's finisher
          // of this row group holds a partial over its K shard.  Publish ours
          // to every rank (this one included) as tagged words; the residual
          // update waits until the phase's last row group was sent (below), so
          // no rank's sends wait on another rank.
          const int set = g.kind == kO ? 0 : 1;
          const uint64_t hi = static_cast<uint64_t>(p.tp_seq_base + seq) << 32;
          const uint64_t w0 = hi | __float_as_uint(v0), w1 = hi | __float_as_uint(v1);
          for (int r = 0; r < p.tp_size; ++r) {
            TpExchange *peer = reinterpret_cast<TpExchange *>(
                __shfl_sync(0xffffffffu, reinterpret_cast<unsigned long long>(peer_mine), r));
            st_relaxed_sys_u64(&peer->part[set][p.tp_rank][n0][b], w0);
            st_relaxed_sys_u64(&peer->part[set][p.tp_rank][n1][b], w1);
          }
        } else if (g.kind == kO || g.kind == kDown) {
          // hidden = residual + materialize(mm_t(x, W))  (:380-386, :399-403)
          p.h[static_cast<size_t>(b) * m.H + n0] = tobf(__fadd_rn(e0, rbf(v0)));
          p.h[static_cast<size_t>(b) * m.H + n1] = tobf(__fadd_rn(e1, rbf(v1)));
        } else if (g.kind == kGU) {
          // silu(bf16(x Wg^T)) * bf16(x Wu^T), each op rounded to bf16 (:391-398);
          // rows 0-7 of the group are gate rows, 8-15 the matching up rows
          const float gate = rbf(v0);
          const float up = rbf(v1);
          const float silu = rbf(__fdiv_rn(gate, __fadd_rn(1.0f, expf(-gate))));
          p.act[static_cast<size_t>(b) * m.I_pad + rg * 8 + (lane >> 2)] = tobf(__fmul_rn(silu, up));
        } else {
          // logits = f32(bf16(x W^T)) (:405-408); first-max argmax partials
          const float l0 = rbf(v0), l1 = rbf(v1);
          float cb = -INFINITY;
          int32_t ci = INT_MAX, cbad = 0;
          // rows of this rank's vocabulary shard; ids are global
          if (n0 < m.Vl) {
            if (p.logits != nullptr) p.logits[(static_cast<size_t>(step) * kBatch + b) * m.V + m.v0 + n0] = l0;
            cbad |= !isfinite(l0);
            if (l0 > cb) { cb = l0; ci = static_cast<int32_t>(m.v0 + n0); }
          }
          if (n1 < m.Vl) {
            if (p.logits != nullptr) p.logits[(static_cast<size_t>(step) * kBatch + b) * m.V + m.v0 + n1] = l1;
            cbad |= !isfinite(l1);
            if (l1 > cb) { cb = l1; ci = static_cast<int32_t>(m.v0 + n1); }
          }
#pragma unroll
          for (int off = 4; off < 32; off <<= 1) {   // lanes sharing b: l ^ 4, 8, 16
            const float ob = __shfl_xor_sync(0xffffffffu, cb, off);
            const int32_t oi = __shfl_xor_sync(0xffffffffu, ci, off);
            cbad |= __shfl_xor_sync(0xffffffffu, cbad, off);
            if (ob > cb || (ob == cb && oi < ci)) { cb = ob; ci = oi; }
          }
          if (cb > best || (cb == best && ci < best_i)) { best = cb; best_i = ci; }
          bad |= cbad;
        }
      }
    }
    if (++kk == tr.KT) { kk = 0; ++rg; }
  }
  if (g.kind == kLM && lane < kBatch) {
    p.arg_val[blockIdx.x * kBatch + lane] = best;
    p.arg_idx[blockIdx.x * kBatch + lane] = best_i;
    p.arg_bad[blockIdx.x * kBatch + lane] = bad;
  }
  if (tp_partial) {
    // hidden = residual + materialize(sum over ranks in rank order) for every
    // row group this CTA finished -- the reference's (:380-386, :399-403) with
    // the sum split over ranks; each word is valid once it carries the tag
    const int set = g.kind == kO ? 0 : 1;
    const uint32_t tag = p.tp_seq_base + seq;
    const uint64_t wait0 = p.trace != nullptr ? globaltimer() : 0;
    const int b = b_lane;
    const int64_t first_head = tr.t0 % tr.KT == 0 ? tr.t0 / tr.KT : tr.t0 / tr.KT + 1;
    for (int64_t r = first_head; tr.t0 < tr.t1 && r * tr.KT < tr.t1; ++r) {
      const int64_t n0 = r * kRows + (lane >> 2), n1 = n0 + 8;
      float sum0 = 0.f, sum1 = 0.f;
      for (int src = 0; src < p.tp_size; ++src) {
        sum0 = __fadd_rn(sum0, tp_recv(p, &p.tp_local->part[set][src][n0][b], tag));
        sum1 = __fadd_rn(sum1, tp_recv(p, &p.tp_local->part[set][src][n1][b], tag));
      }
      float e0, e1;
      if (r == pa_rg) {
        e0 = pa0;
        e1 = pa1;
      } else if (r == pb_rg) {
        e0 = pb0;
        e1 = pb1;
      } else {
        e0 = bf(__ldcg(p.h + static_cast<size_t>(b) * m.H + n0));
        e1 = bf(__ldcg(p.h + static_cast<size_t>(b) * m.H + n1));
      }
      p.h[static_cast<size_t>(b) * m.H + n0] = tobf(__fadd_rn(e0, rbf(sum0)));
      p.h[static_cast<size_t>(b) * m.H + n1] = tobf(__fadd_rn(e1, rbf(sum1)));
    }
    if (p.trace != nullptr && blockIdx.x == 0 && lane == 0 && trace_slot < kTraceMax)
      p.trace[5 * kTraceMax + trace_slot] = globaltimer() - wait0;
  }
  if (mark != nullptr && lane == 0) {
    mark[5] = static_cast<uint32_t>(partner_ns);
    mark[6] = static_cast<uint32_t>(globaltimer());
  }
  // The phase's outputs become visible GPU-wide through the chain: this
  // warp's writes -> __syncwarp -> lane 0's mbarrier arrive (release, CTA
  // scope) -> thread 0's wait on it (acquire, CTA scope) -> the consumers'
  // bar.sync -> thread 0's release add at the grid barrier (GPU scope,
  // cumulative) -> every other CTA's acquire load of the barrier counter.
  __syncwarp();
  if (mark != nullptr && lane == 0) mark[7] = static_cast<uint32_t>(globaltimer());
  if (lane == 0) mbar_arrive(s.phase_done);
}

// Epilogue warp main loop: follows the projection phases of every step.
__device__ void epilogue_main(const EpochParams &p, const Smem &s) {
  const int lane = threadIdx.x & 31;
  const int L = p.m.L;
  const int phases = 5 * L + 2;
  RingCursor red;
  for (int step = 0; step < kMaxSteps; ++step) {
    bool go = true;
    if (lane == 0) go = wait_step(p, s, step);
    go = __shfl_sync(0xffffffffu, go ? 1 : 0, 0) != 0;
    if (!go) return;
    for (int ph = 0; ph < phases; ++ph) {
      const int kind = gemv_kind_of_phase(ph, L);
      if (kind < 0) continue;
      const int seq = step * phases + ph + 1;
      // never finish a phase before the consumers started it
      bool started = true;
      if (lane == 0) {
        const uint64_t deadline = globaltimer() + p.timeout_ns;
        for (uint32_t polls = 1; *s.phase_started < seq; ++polls) {
          if ((polls & 15) == 0 && (*s.prod_ctl == -1 || aborted(p) || globaltimer() > deadline)) {
            started = false;
            break;
          }
        }
      }
      started = __shfl_sync(0xffffffffu, started ? 1 : 0, 0) != 0;
      if (!started) return;
      const Gemv g = make_gemv(p, ph / 5, kind);
      gemv_finish(p, s, g, red, static_cast<uint32_t>(seq), step,
                  static_cast<uint32_t>(*reinterpret_cast<volatile int32_t *>(&s.misc[12])));
    }
  }
}

// ---- consumer: paged GQA decode attention ---------------------------------------------------------
// One unit per (row, query head), units spread over CTAs.  RoPE on q and k
// (:231-240), the new k/v written at slot[row] for active rows (:242-264),
// scores bf16(q.K) then bf16(s / sqrt(d)), softmax in fp32 rounded to bf16,
// output bf16(P.V) (:334-379).  Positions >= seq_len contribute exactly zero in
// the reference (masked to bf16.min), so they are skipped.
//
// Latency layout: a unit is one dependent trip to memory.  Together with the
// q/k/v loads every thread issues its cached K row (scores pass: thread t owns
// position t of a 256-position chunk) and, with cp.async into the free part of
// the scratch, the V slices it consumes in the P.V pass (thread = position
// group x 8-dim slice) for the first positions that fit; the row state and the
// block table come from shared memory.  Longer contexts load the remaining K
// chunks and V rows in their loops.
constexpr int kAttnChunk = kConsumerThreads;   // positions per scores chunk

template <int D>
__host__ __device__ constexpr int attn_groups() { return kConsumerThreads / (D / 8); }

// Shared scratch of one attention unit: qf[D] f32, kn[D] + vn[D] bf16, sc[C]
// f32, rd[16] f32, part[groups][D] f32; the staged V rows follow.
__host__ __device__ inline size_t attn_scratch_bytes(int D, int C) {
  const int groups = kConsumerThreads / (D / 8);
  return static_cast<size_t>(D) * 4 + static_cast<size_t>(D) * 4 + static_cast<size_t>((C + 3) & ~3) * 4 +
         16 * 4 + static_cast<size_t>(groups) * D * 4;
}

// Waits (thread 0, bounded) until KV head `kvh`'s QKV row groups of the
// current QKV phase are all written, then makes them visible to the CTA.
__device__ __forceinline__ void wait_qkv_group(const EpochParams &p, const Smem &s, int kvh, uint32_t target) {
  if (threadIdx.x == 0) {
    const uint32_t *counter = &p.sync->qkv_done[kvh][0];
    if (static_cast<int32_t>(ld_acquire_u32(counter) - target) < 0) {
      const uint64_t deadline = globaltimer() + p.timeout_ns;
      uint32_t polls = 0;
      while (static_cast<int32_t>(ld_acquire_u32(counter) - target) < 0) {
        if ((++polls & 15) == 0) {
          if (aborted(p)) break;
          if (globaltimer() > deadline) { raise_error(p, 1005); break; }
        }
      }
    }
  }
  named_sync(1, kConsumerThreads);
}

template <int D>
__device__ void attention_phase_d(const EpochParams &p, const Smem &s, int layer, uint32_t qkv_target) {
  const ModelDims &m = p.m;
  const int tid = threadIdx.x;
  constexpr int half = D / 2;
  constexpr int kSlices = D / 8;                 // 16-byte slices of a K/V row
  constexpr int kGroups = attn_groups<D>();      // position groups of the P.V pass
  const int groups = m.nq / m.nkv;
  float *qf = reinterpret_cast<float *>(s.xs);         // [D]  roped q (bf16 values)
  bf16 *kn = reinterpret_cast<bf16 *>(qf + D);          // [D]  roped new k
  bf16 *vn = kn + D;                                    // [D]  new v
  float *sc = reinterpret_cast<float *>(vn + D);        // [C]  scores, then probabilities
  float *rd = sc + ((m.C + 3) & ~3);                    // [16] reductions
  float *part = rd + 16;                                // [groups][D] P.V partials
  bf16 *vs = reinterpret_cast<bf16 *>(reinterpret_cast<uint8_t *>(s.xs) + attn_scratch_bytes(D, m.C));
  // positions whose V rows are staged in shared memory
  const size_t scratch = static_cast<size_t>(kBatch) * p.xs_stride * 2 +
                         static_cast<size_t>(kRedSlots) * kConsumerWarps * 64 * 4;
  const int vcap = static_cast<int>(min(static_cast<size_t>(m.C), (scratch - attn_scratch_bytes(D, m.C)) / (D * 2)));
  if (layer == 0) {   // the row state is constant over the layers of a step
    if (tid < kBatch) {
      s.row_pos[tid] = __ldcg(&p.work->position[tid]);
      s.row_len[tid] = __ldcg(&p.work->length[tid]);
      s.row_slot[tid] = __ldcg(&p.work->slot[tid]);
      s.row_act[tid] = __ldcg(&p.work->active[tid]);
    }
    named_sync(1, kConsumerThreads);
  }
  const size_t layer_off = static_cast<size_t>(layer) * m.NB * m.bs * m.nkv * D;
  const size_t row_stride = static_cast<size_t>(m.nkv) * D;   // elements between cache slots
  const int units = kBatch * m.nq;
  const int warp = tid >> 5, lane = tid & 31;
  const int vslice = tid % kSlices, vgroup = tid / kSlices;
  for (int u = blockIdx.x; u < units; u += p.grid) {
    const int b = u / m.nq, qh = u % m.nq, kvh = qh / groups;
    bf16 *out = p.attn + static_cast<size_t>(b) * m.Kq + qh * D;
    if (s.row_act[b] == 0) {
      for (int i = tid; i < D; i += kConsumerThreads) out[i] = tobf(0.f);
      continue;
    }
    const int64_t pos = s.row_pos[b];
    const int len = s.row_len[b];
    const int slot = s.row_slot[b];
    const bf16 *kcache = p.key_cache + layer_off + kvh * D;
    const bf16 *vcache = p.value_cache + layer_off + kvh * D;
    // a cached row of position t (never the new position: its k/v come from
    // shared memory); nullptr outside the row's valid blocks
    auto cached = [&](const bf16 *base, int t) -> const uint4 * {
      const int st = slot_in_row(m, s.bt, b, t);
      return st < 0 ? nullptr : reinterpret_cast<const uint4 *>(base + static_cast<size_t>(st) * row_stride);
    };
    auto load_k = [&](uint4 (&krow)[kSlices], int c0) {
      const int t = c0 + tid;
      const uint4 *src = (t < len && t != pos) ? cached(kcache, t) : nullptr;
#pragma unroll
      for (int i = 0; i < kSlices; ++i) krow[i] = src != nullptr ? __ldcg(src + i) : make_uint4(0, 0, 0, 0);
    };
    uint4 krow[kSlices];
    load_k(krow, 0);
    const int vstaged = min(len, vcap);
    for (int t = vgroup; t < vstaged; t += kGroups) {
      if (t == pos) continue;
      const uint4 *src = cached(vcache, t);
      bf16 *dst = vs + static_cast<size_t>(t) * D + vslice * 8;
      if (src != nullptr) {
        cp_async16(dst, src + vslice);
      } else {
        *reinterpret_cast<uint4 *>(dst) = make_uint4(0, 0, 0, 0);
      }
    }
    cp_async_commit();
    // the cached rows above do not depend on this layer's projections; q, k, v do
    wait_qkv_group(p, s, kvh, qkv_target);
    const bf16 *qsrc = p.qkv + static_cast<size_t>(b) * m.Nqkv + qh * D;
    const bf16 *ksrc = p.qkv + static_cast<size_t>(b) * m.Nqkv + m.Hq + kvh * D;
    const bf16 *vsrc = p.qkv + static_cast<size_t>(b) * m.Nqkv + m.Hq + m.nkv * D + kvh * D;
    const bf16 *cs = p.rope_cos + pos * D;
    const bf16 *sn = p.rope_sin + pos * D;
    if (tid < D) {
      const int i = tid;
      const float c = bf(cs[i]), sv = bf(sn[i]);
      const float q = bf(__ldcg(qsrc + i));
      const float qr = i < half ? -bf(__ldcg(qsrc + i + half)) : bf(__ldcg(qsrc + i - half));
      qf[i] = rbf(__fadd_rn(rbf(__fmul_rn(q, c)), rbf(__fmul_rn(qr, sv))));
      const float k = bf(__ldcg(ksrc + i));
      const float kr = i < half ? -bf(__ldcg(ksrc + i + half)) : bf(__ldcg(ksrc + i - half));
      kn[i] = tobf(__fadd_rn(rbf(__fmul_rn(k, c)), rbf(__fmul_rn(kr, sv))));
      vn[i] = __ldcg(vsrc + i);
    }
    named_sync(1, kConsumerThreads);
    if (qh % groups == 0 && slot >= 0 && slot < m.NB * m.bs && tid < D) {
      const size_t off = layer_off + (static_cast<size_t>(slot) * m.nkv + kvh) * D;
      p.key_cache[off + tid] = kn[tid];
      p.value_cache[off + tid] = vn[tid];
    }
    // scores: thread t owns position t of each chunk
    float local_max = -INFINITY;
    for (int c0 = 0; c0 < len; c0 += kAttnChunk) {
      if (c0 > 0) load_k(krow, c0);
      const int t = c0 + tid;
      if (t < len) {
        if (t == pos) {
#pragma unroll
          for (int i = 0; i < kSlices; ++i) krow[i] = reinterpret_cast<const uint4 *>(kn)[i];
        }
        float dot = 0.f;
#pragma unroll
        for (int i = 0; i < kSlices; ++i) {
          const __nv_bfloat162 *k2 = reinterpret_cast<const __nv_bfloat162 *>(&krow[i]);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float2 kf = __bfloat1622float2(k2[j]);
            dot = fmaf(qf[8 * i + 2 * j], kf.x, dot);
            dot = fmaf(qf[8 * i + 2 * j + 1], kf.y, dot);
          }
        }
        const float s2 = rbf(__fdiv_rn(rbf(dot), m.sqrt_d));
        sc[t] = s2;
        local_max = fmaxf(local_max, s2);
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1)
      local_max = fmaxf(local_max, __shfl_xor_sync(0xffffffffu, local_max, off));
    if (lane == 0) rd[warp] = local_max;
    named_sync(1, kConsumerThreads);
    float mx = rd[0];
#pragma unroll
    for (int w = 1; w < kConsumerWarps; ++w) mx = fmaxf(mx, rd[w]);
    float local_sum = 0.f;
    for (int t = tid; t < len; t += kConsumerThreads) {
      const float e = expf(__fsub_rn(sc[t], mx));
      sc[t] = e;
      local_sum += e;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) local_sum += __shfl_xor_sync(0xffffffffu, local_sum, off);
    if (lane == 0) rd[8 + warp] = local_sum;
    named_sync(1, kConsumerThreads);
    float sum = 0.f;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) sum += rd[8 + w];
    for (int t = tid; t < len; t += kConsumerThreads) sc[t] = rbf(__fdiv_rn(sc[t], sum));
    named_sync(1, kConsumerThreads);
    // output: this thread accumulates dims [8*vslice, 8*vslice+8) over the
    // positions vgroup + kGroups*i in ascending order (its own staged V slices,
    // then four rows at a time from memory beyond the staged ones)
    float o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = 0.f;
    auto accumulate = [&](const uint4 &v4, float pr) {
      const __nv_bfloat162 *v2 = reinterpret_cast<const __nv_bfloat162 *>(&v4);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 vf = __bfloat1622float2(v2[j]);
        o[2 * j] = fmaf(pr, vf.x, o[2 * j]);
        o[2 * j + 1] = fmaf(pr, vf.y, o[2 * j + 1]);
      }
    };
    const uint4 vnew = reinterpret_cast<const uint4 *>(vn)[vslice];
    cp_async_wait_all();
    int t = vgroup;
    for (; t < vstaged; t += kGroups)
      accumulate(t == pos ? vnew : lds128(vs + static_cast<size_t>(t) * D + vslice * 8), sc[t]);
    for (; t < len; t += 4 * kGroups) {
      uint4 vv[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int tq = t + q * kGroups;
        const uint4 *src = (tq < len && tq != pos) ? cached(vcache, tq) : nullptr;
        vv[q] = tq == pos ? vnew : (src != nullptr ? __ldcg(src + vslice) : make_uint4(0, 0, 0, 0));
      }
#pragma unroll
      for (int q = 0; q < 4; ++q)
        if (t + q * kGroups < len) accumulate(vv[q], sc[t + q * kGroups]);
    }
    float4 *dst = reinterpret_cast<float4 *>(part + vgroup * D + vslice * 8);
    dst[0] = make_float4(o[0], o[1], o[2], o[3]);
    dst[1] = make_float4(o[4], o[5], o[6], o[7]);
    named_sync(1, kConsumerThreads);
    if (tid < D) {
      float total = 0.f;
#pragma unroll
      for (int g2 = 0; g2 < kGroups; ++g2) total += part[g2 * D + tid];
      out[tid] = tobf(total);
    }
    named_sync(1, kConsumerThreads);
  }
}

__device__ void attention_phase(const EpochParams &p, const Smem &s, int layer, uint32_t qkv_target) {
  if (p.m.d == 128) {
    attention_phase_d<128>(p, s, layer, qkv_target);
  } else {
    attention_phase_d<64>(p, s, layer, qkv_target);
  }
}

// ---- consumer: epoch prologue (CTA 0, thread 0) ---------------------------------------------------
// Decodes the control vector and validates every input exactly like the
// reference controller (:207-241, :335-385).  Returns the fallback status or 0.
__device__ int32_t validate_inputs(const EpochParams &p) {
  const ModelDims &m = p.m;
  EpochIO *io = p.io;
  EpochWork *w = p.work;
  const int32_t encoded = io->control[2 + kBatch];
  const bool importing = (encoded & kImportFlag) != 0;
  w->importing = importing;
  const int32_t mask = importing ? (encoded & (kImportFlag - 1)) : 0;
  w->variant = importing ? (encoded & ~(kImportFlag | 0xF)) : encoded;
  w->max_steps = io->control[0];
  w->sampling = io->control[1 + kBatch];
  w->import_rows = 0;
  w->checksum = 0;
  w->model_calls = 0;
  for (int b = 0; b < kBatch; ++b) {
    w->eos[b] = io->control[1 + b];
    w->generation[b] = io->control[3 + kBatch + b];
    w->token[b] = io->token[b];
    w->position[b] = io->position[b];
    w->length[b] = io->seq_len[b];
    w->active[b] = io->active[b];
    w->active0[b] = io->active[b];
    w->executed[b] = 0;
    w->reason[b] = kNone;
    w->new_gen[b] = 0;
  }
  for (int i = 0; i < kBatch * m.bpr; ++i) w->bt[i] = io->block_table[i];
  for (int b = 0; b < kBatch; ++b)
    w->slot[b] = importing ? compute_slot(m, w->bt, b, w->position[b]) : io->slot[b];
  for (int i = 0; i < kMaxSteps * kBatch; ++i) io->history[i] = -1;

  if (w->max_steps < 1 || w->max_steps > kMaxSteps || w->sampling != 0 || w->variant != 0) {
    if (w->sampling != 0) return kUnsupportedSampling;
    if (w->variant != 0) return kUnsupportedGraph;
    return kInvalidMetadata;
  }
  for (int b = 0; b < kBatch; ++b)
    if (w->eos[b] < 0 || w->eos[b] >= m.V) return kInvalidMetadata;
  unsigned long long seen[4] = {0ull, 0ull, 0ull, 0ull};
  for (int i = 0; i < kBatch * m.bpr; ++i) {
    const int blk = w->bt[i];
    if (blk < 0 || blk >= m.NB || blk >= 256) return kInvalidBlockTable;
    const unsigned long long bit = 1ull << (blk & 63);
    if (seen[blk >> 6] & bit) return kInvalidBlockTable;
    seen[blk >> 6] |= bit;
  }
  for (int b = 0; b < kBatch; ++b) {
    const int32_t a = w->active0[b];
    if ((a != 0 && a != 1) || w->token[b] < 0 || w->token[b] >= m.V || w->position[b] < 0 ||
        w->position[b] >= m.C)
      return kInvalidMetadata;
    if (a == 1) {
      if (w->generation[b] <= 0) return kInvalidMetadata;
      if (w->length[b] != w->position[b] + 1) return kInvalidMetadata;
      if (w->position[b] + w->max_steps > m.C) return kCapacityExceeded;
    } else if (w->length[b] == 0) {
      if (w->generation[b] != 0) return kInvalidMetadata;
      w->reason[b] = kEmpty;
    } else if (w->length[b] == w->position[b] + 1) {
      w->reason[b] = kAlreadyFinished;
    } else {
      return kInvalidMetadata;
    }
    if (compute_slot(m, w->bt, b, w->position[b]) != w->slot[b]) return kSlotMismatch;
  }
  if (importing) {
    if (mask <= 0 || mask >= (1 << kBatch)) return kInvalidMetadata;
    // rows are imported in order; the first invalid row stops the import (:395-400)
    for (int b = 0; b < kBatch; ++b) {
      if ((mask & (1 << b)) == 0) continue;
      if (w->active0[b] != 1 || w->generation[b] <= 0) return -kInvalidMetadata;  // partial import
      w->import_rows |= 1 << b;
    }
  }
  return kOk;
}

// Sum and position-weighted sum of one block for Adler-32 (mod 65521 on
// combine): S1 = sum d_i, S2 = sum (n - i + 1) d_i, i = 1..n.
__device__ void adler_block(const uint8_t *data, int n, uint64_t &S1, uint64_t &S2, float *scratch) {
  const int tid = threadIdx.x;
  const int per = n / kConsumerThreads;
  const uint8_t *mine = data + static_cast<size_t>(tid) * per;
  uint64_t s1 = 0, w = 0;
  for (int i = 0; i < per; i += 16) {
    const uint4 v = __ldcg(reinterpret_cast<const uint4 *>(mine + i));
    const uint8_t *bytes = reinterpret_cast<const uint8_t *>(&v);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      s1 += bytes[j];
      w += static_cast<uint64_t>(per - (i + j)) * bytes[j];
    }
  }
  const uint64_t tail = static_cast<uint64_t>(n) - static_cast<uint64_t>(tid + 1) * per;
  uint64_t s2 = w + tail * s1;
  // block reduction of (s1, s2) through shared memory (scratch holds 2*256 u64)
  uint64_t *red = reinterpret_cast<uint64_t *>(scratch);
  red[tid] = s1;
  red[kConsumerThreads + tid] = s2;
  named_sync(1, kConsumerThreads);
  if (tid == 0) {
    uint64_t a = 0, c = 0;
    for (int i = 0; i < kConsumerThreads; ++i) {
      a += red[i];
      c += red[kConsumerThreads + i];
    }
    S1 = a;
    S2 = c;
  }
  named_sync(1, kConsumerThreads);
}

// ---- consumer: decoder-step prologue (CTA 0, thread 0) ------------------------------------------------
// One call of the 9-in / 4-out decoder ABI: the inputs become the working row
// state of a single step with no controller checks (the host validated the
// ranges the kernel indexes with), no import and no continuity.
__device__ void decoder_step_setup(const EpochParams &p) {
  EpochWork *w = p.work;
  EpochIO *io = p.io;
  w->importing = 0;
  w->variant = 0;
  w->sampling = 0;
  w->max_steps = 1;
  w->import_rows = 0;
  w->checksum = 0;
  w->model_calls = 0;
  for (int b = 0; b < kBatch; ++b) {
    w->eos[b] = -1;
    w->generation[b] = 0;
    w->token[b] = io->token[b];
    w->position[b] = io->position[b];
    w->length[b] = io->seq_len[b];
    w->slot[b] = io->slot[b];
    w->active[b] = io->active[b];
    w->active0[b] = io->active[b];
    w->executed[b] = 0;
    w->reason[b] = kNone;
    w->new_gen[b] = 0;
  }
  for (int i = 0; i < kBatch * p.m.bpr; ++i) w->bt[i] = io->block_table[i];
  for (int i = 0; i < kMaxSteps * kBatch; ++i) io->history[i] = -1;
  w->status = kOk;
  w->stop = 0;
}

// ---- the kernel ---------------------------------------------------------------------------------------
// The register file is split over the SM's four sub-partitions (16K registers each) and ten warps put
// three warps on two of them, so one CTA of 320 threads fits only at <= 168 registers per thread; the
// launch bound makes ptxas hold that ceiling (a higher cap compiles but leaves zero resident CTAs).
__global__ void __launch_bounds__(kThreads, 1) resident_epoch_kernel(const EpochParams p) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  const Smem s = carve_smem(smem_raw, p);
  const int tid = threadIdx.x;
  const ModelDims &m = p.m;
  EpochWork *w = p.work;
  EpochIO *io = p.io;

  if (tid == 0) {
    for (int i = 0; i < p.stages; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], kConsumerWarps);
    }
    for (int i = 0; i < kRedSlots; ++i) {
      mbar_init(&s.red_full[i], kConsumerWarps);
      mbar_init(&s.red_empty[i], 1);
    }
    mbar_init(s.phase_done, 1);
    *s.prod_ctl = -2;        // producer and epilogue warps wait for "step 0 go"
    *s.phase_started = 0;
    mbar_fence_init();
  }
  __syncthreads();
  const int warp_id = tid >> 5;
  if (warp_id == kProducerWarp) {
    producer_main(p, s);
    return;
  }
  if (warp_id == kEpilogueWarp) {
    epilogue_main(p, s);
    return;
  }

  uint32_t barrier_index = 0;
  RingCursor ring, red;
  uint32_t done_parity = 0;
  bool ok = true;
  const size_t block_elems = static_cast<size_t>(m.bs) * m.nkv * m.d;
  const size_t payload_block_elems = static_cast<size_t>(m.bs) * m.nkv_all * m.d;
  const size_t layer_elems = static_cast<size_t>(m.NB) * block_elems;

  const bool step_mode = p.mode == kModeDecoderStep;
  // 1. validation (CTA 0)
  if (blockIdx.x == 0 && tid == 0 && step_mode) {
    decoder_step_setup(p);
  } else if (blockIdx.x == 0 && tid == 0) {
    int32_t st = validate_inputs(p);
    if (st < 0) {   // an imported row failed its check after earlier rows were imported
      w->status = -st;
    } else {
      w->status = st;
      if (st != kOk) w->import_rows = 0;
    }
    w->stop = w->status != kOk ? 1 : 0;
  }
  ok = grid_barrier(p, s, ++barrier_index, 1);

  // 2. import: copy the payload block of each imported row into its first
  //    block, zero its other blocks (:387-418); then the Adler-32 proof.
  if (ok && __ldcg(&w->import_rows) != 0) {
    const int rows = __ldcg(&w->import_rows);
    const int units = 2 * m.L * kBatch * m.bpr;
    for (int u = blockIdx.x; u < units; u += p.grid) {
      const int j = u % m.bpr;
      const int b = (u / m.bpr) % kBatch;
      const int layer = (u / (m.bpr * kBatch)) % m.L;
      const int cache = u / (m.bpr * kBatch * m.L);
      if ((rows & (1 << b)) == 0) continue;
      bf16 *dst = (cache == 0 ? p.key_cache : p.value_cache) + layer * layer_elems +
                  static_cast<size_t>(w->bt[b * m.bpr + j]) * block_elems;
      uint4 *d4 = reinterpret_cast<uint4 *>(dst);
      const size_t n16 = block_elems * 2 / 16;
      if (j == 0) {
        // the payload block holds every KV head of the model; this rank copies
        // its heads [kv0, kv0 + nkv) of each slot
        const uint4 *s4 = reinterpret_cast<const uint4 *>(
            p.import_payload +
            ((static_cast<size_t>(cache) * m.L + layer) * kBatch + b) * payload_block_elems * 2);
        const size_t u_loc = static_cast<size_t>(m.nkv) * m.d / 8, u_all = static_cast<size_t>(m.nkv_all) * m.d / 8;
        const size_t u_off = static_cast<size_t>(m.kv0) * m.d / 8;
        for (size_t i = tid; i < n16; i += kConsumerThreads)
          d4[i] = __ldcg(s4 + (i / u_loc) * u_all + u_off + i % u_loc);
      } else {
        for (size_t i = tid; i < n16; i += kConsumerThreads) d4[i] = make_uint4(0, 0, 0, 0);
      }
    }
    if (blockIdx.x == 0 && tid == 0) {
      for (int b = 0; b < kBatch; ++b) {
        if ((rows & (1 << b)) == 0) continue;
        p.res->generation[b] = w->generation[b];
        p.res->token[b] = w->token[b];
        p.res->position[b] = w->position[b];
        p.res->length[b] = w->length[b];
        p.res->valid[b] = 1;
      }
    }
    ok = grid_barrier(p, s, ++barrier_index, 2);
    if (ok && __ldcg(&w->status) == kOk) {
      // blocks in checksum order: K then V, layer-major, row-minor (:419-432)
      int nrows = 0;
      int order[kBatch];
      for (int b = 0; b < kBatch; ++b)
        if (rows & (1 << b)) order[nrows++] = b;
      const int units2 = 2 * m.L * nrows;
      // the imported blocks are the payload's blocks (every KV head): the proof
      // is computed from the device copy of the payload
      const int n = static_cast<int>(payload_block_elems * 2);
      for (int u = blockIdx.x; u < units2; u += p.grid) {
        const int cache = u / (m.L * nrows);
        const int layer = (u / nrows) % m.L;
        const int b = order[u % nrows];
        const uint8_t *src = p.import_payload +
                             ((static_cast<size_t>(cache) * m.L + layer) * kBatch + b) * payload_block_elems * 2;
        uint64_t S1 = 0, S2 = 0;
        adler_block(src, n, S1, S2, reinterpret_cast<float *>(s.xs));
        if (tid == 0) {
          w->adler[2 * u] = S1;
          w->adler[2 * u + 1] = S2;
        }
      }
      ok = grid_barrier(p, s, ++barrier_index, 3);
      if (ok && blockIdx.x == 0 && tid == 0) {
        const uint64_t M = 65521;
        uint64_t a = 1, c = 0;
        for (int u = 0; u < units2; ++u) {
          const uint64_t S1 = __ldcg(&w->adler[2 * u]) % M;
          const uint64_t S2 = __ldcg(&w->adler[2 * u + 1]) % M;
          c = (c + (static_cast<uint64_t>(n) % M) * a + S2) % M;
          a = (a + S1) % M;
        }
        w->checksum = static_cast<uint32_t>((c << 16) | a);
      }
    }
  }

  // 3. generation continuity (:448-473), then clear the rows of new generations
  if (ok && !step_mode && blockIdx.x == 0 && tid == 0 && w->status == kOk) {
    for (int b = 0; b < kBatch && w->status == kOk; ++b) {
      if (w->active0[b] == 0) continue;
      if (p.res->generation[b] == w->generation[b]) {
        if (p.res->valid[b] == 0 || p.res->token[b] != w->token[b] ||
            p.res->position[b] != w->position[b] || p.res->length[b] != w->length[b])
          w->status = kResidentContinuity;
      } else {
        if (w->position[b] != 0 || w->length[b] != 1) w->status = kResidentContinuity;
        w->new_gen[b] = 1;
      }
    }
    if (w->status != kOk) {
      for (int b = 0; b < kBatch; ++b) w->new_gen[b] = 0;
    }
    w->stop = w->status != kOk ? 1 : 0;
  }
  if (ok) ok = grid_barrier(p, s, ++barrier_index, 4);
  // the validated block table, read by the attention units of every step
  for (int i = tid; i < kBatch * m.bpr; i += kConsumerThreads) s.bt[i] = __ldcg(&w->bt[i]);
  if (ok && __ldcg(&w->status) == kOk) {
    bool any = false;
    for (int b = 0; b < kBatch; ++b) any |= __ldcg(&w->new_gen[b]) != 0;
    if (any) {
      const int units = 2 * m.L * kBatch * m.bpr;
      for (int u = blockIdx.x; u < units; u += p.grid) {
        const int j = u % m.bpr;
        const int b = (u / m.bpr) % kBatch;
        const int layer = (u / (m.bpr * kBatch)) % m.L;
        const int cache = u / (m.bpr * kBatch * m.L);
        if (!__ldcg(&w->new_gen[b])) continue;
        bf16 *dst = (cache == 0 ? p.key_cache : p.value_cache) + layer * layer_elems +
                    static_cast<size_t>(w->bt[b * m.bpr + j]) * block_elems;
        uint4 *d4 = reinterpret_cast<uint4 *>(dst);
        for (size_t i = tid; i < block_elems * 2 / 16; i += kConsumerThreads) d4[i] = make_uint4(0, 0, 0, 0);
      }
      ok = grid_barrier(p, s, ++barrier_index, 5);
    }
  }

  // 4. the K-loop (:485-591)
  const int L = m.L;
  const int phases = 5 * L + 2;
  for (int step = 0; ok && step < kMaxSteps; ++step) {
    if (__ldcg(&w->stop)) break;
    if (tid == 0) *s.prod_ctl = step;   // release the producer for this step
    for (int ph = 0; ok && ph < phases; ++ph) {
      const uint32_t seq = static_cast<uint32_t>(step * phases + ph + 1);
      const int kind = gemv_kind_of_phase(ph, L);
      if (kind >= 0) {
        const Gemv g = make_gemv(p, ph / 5, kind);
        if (tid == 0) {
          s.misc[12] = static_cast<int32_t>(barrier_index + 1);   // the phase's trace slot
          __threadfence_block();
          *s.phase_started = static_cast<int>(seq);
        }
        gemv_consume(p, s, g, ring, red, barrier_index + 1);
        // the epilogue warp has written every output of the phase
        if (tid == 0) wait_bar(p, s.phase_done, done_parity, nullptr, 1004);
        done_parity ^= 1u;
      } else if (ph < 5 * L) {
        // attention follows QKV without a grid barrier: this CTA's epilogue
        // warp is done with the shared memory the attention scratch reuses,
        // and each unit waits for its own KV head's row groups
        named_sync(1, kConsumerThreads);
        attention_phase(p, s, ph / 5, qkv_rows_per_group(m) * static_cast<uint32_t>(step * L + ph / 5 + 1));
      } else if (blockIdx.x == 0 && step_mode) {
        // the decoder ABI's fourth output: next_position = where(active, pos + 1, pos)
        // (batched_decoder_step.py:409-411), in the history words
        if (tid == 0) {
          w->model_calls = 1;
          for (int b = 0; b < kBatch; ++b) io->history[b] = w->active[b] ? w->position[b] + 1 : w->position[b];
          w->stop = 1;
        }
      } else if (blockIdx.x == 0) {
        // control: two-pass argmax (pass 2 over the per-CTA partials), then the
        // per-row bookkeeping of the reference K-loop body (:537-591)
        {
          // two warps per row: lane-strided over the CTA partials, then shuffles
          const int lm_ctas = static_cast<int>(m.V_pad / kRows < p.grid ? m.V_pad / kRows : p.grid);
          const int b = tid >> 6, sub = tid & 63;
          float best = -INFINITY;
          int32_t idx = INT_MAX, bad = 0;
          for (int c = sub; c < lm_ctas; c += 64) {
            const float v = __ldcg(&p.arg_val[c * kBatch + b]);
            const int32_t i = __ldcg(&p.arg_idx[c * kBatch + b]);
            bad |= __ldcg(&p.arg_bad[c * kBatch + b]);
            if (v > best || (v == best && i < idx)) { best = v; idx = i; }
          }
#pragma unroll
          for (int off = 16; off > 0; off >>= 1) {
            const float ob = __shfl_xor_sync(0xffffffffu, best, off);
            const int32_t oi = __shfl_xor_sync(0xffffffffu, idx, off);
            bad |= __shfl_xor_sync(0xffffffffu, bad, off);
            if (ob > best || (ob == best && oi < idx)) { best = ob; idx = oi; }
          }
          if ((tid & 31) == 0) {
            s.best_val[tid >> 5] = best;
            s.best_idx[tid >> 5] = idx;
            s.best_bad[tid >> 5] = bad;
          }
          named_sync(1, kConsumerThreads);
          if (tid < kBatch) {
            const int w0 = 2 * tid, w1 = 2 * tid + 1;
            const bool second = s.best_val[w1] > s.best_val[w0] ||
                                (s.best_val[w1] == s.best_val[w0] && s.best_idx[w1] < s.best_idx[w0]);
            s.misc[4 + tid] = second ? s.best_idx[w1] : s.best_idx[w0];
            s.misc[8 + tid] = s.best_bad[w0] | s.best_bad[w1];
            if (p.tp_size > 1) {
              // this rank's vocabulary shard result, sent to every rank
              TpArg a;
              a.val = second ? s.best_val[w1] : s.best_val[w0];
              a.idx = s.misc[4 + tid];
              a.bad = s.misc[8 + tid];
              a.pad = 0;
              for (int r = 0; r < p.tp_size; ++r) p.tp_peer[r]->arg[p.tp_rank][tid] = a;
              __threadfence_system();
            }
          }
          named_sync(1, kConsumerThreads);
        }
        if (p.tp_size > 1) {
          // cross-rank pass: first maximum over the ranks' shards in rank order
          // (shards are in increasing id order, so ties keep the lowest id)
          if (threadIdx.x < 32) {
            const int lane = threadIdx.x;
            if (lane < p.tp_size) st_release_sys_u32(&p.tp_peer[lane]->flag[p.tp_rank][0], p.tp_seq_base + seq);
            int ready = 1;
            if (lane < p.tp_size) {
              const uint32_t *flag = &p.tp_local->flag[lane][0];
              const uint64_t deadline = globaltimer() + p.timeout_ns;
              uint32_t polls = 0;
              while (static_cast<int32_t>(ld_acquire_sys_u32(flag) - (p.tp_seq_base + seq)) < 0) {
                if ((++polls & 15) == 0) {
                  if (aborted(p)) { ready = 0; break; }
                  if (globaltimer() > deadline) { raise_error(p, 401); ready = 0; break; }
                }
              }
            }
            ready = __all_sync(0xffffffffu, ready);
            if (lane == 0) s.misc[1] = ready;
          }
          named_sync(1, kConsumerThreads);
          if (tid < kBatch && s.misc[1]) {
            float bv = -INFINITY;
            int32_t bi = INT_MAX, bb = 0;
            for (int r = 0; r < p.tp_size; ++r) {
              const int4 raw = __ldcg(reinterpret_cast<const int4 *>(&p.tp_local->arg[r][tid]));
              const float v = __int_as_float(raw.x);
              bb |= raw.z;
              if (v > bv || (v == bv && raw.y < bi)) { bv = v; bi = raw.y; }
            }
            s.misc[4 + tid] = bi;
            s.misc[8 + tid] = bb;
          }
          named_sync(1, kConsumerThreads);
        }
        if (tid == 0) {
          const int calls = ++w->model_calls;
          const int st = calls - 1;
          for (int b = 0; b < kBatch; ++b) {
            if (w->active[b] == 0) continue;   // position stays (:547-552)
            const int64_t forced = io->use_forced ? io->forced[st * kBatch + b] : -1;
            if (forced >= m.V) { w->status = kInvalidMetadata; break; }   // next embedding row must exist
            if (forced < 0 && s.misc[8 + b]) { w->status = kNonFiniteLogits; break; }
            const int64_t tok = forced >= 0 ? forced : s.misc[4 + b];
            io->history[st * kBatch + b] = tok;
            ++w->executed[b];
            w->position[b] += 1;
            w->token[b] = tok;
            w->length[b] = static_cast<int32_t>(w->position[b] + 1);
            if (w->position[b] == m.C) {
              w->slot[b] = -1;
            } else {
              const int sl = compute_slot(m, w->bt, b, w->position[b]);
              if (sl < 0) { w->status = kCapacityExceeded; break; }
              w->slot[b] = sl;
            }
            if (tok == w->eos[b]) {
              w->active[b] = 0;
              w->reason[b] = kEos;
            }
          }
          int any = 0;
          for (int b = 0; b < kBatch; ++b) any |= w->active[b];
          w->stop = (w->status != kOk || calls >= w->max_steps || any == 0) ? 1 : 0;
          if (p.stream != nullptr && w->status == kOk) {
            // streaming egress: this step's tokens, then the step count
            for (int b = 0; b < kBatch; ++b)
              *reinterpret_cast<volatile int64_t *>(&p.stream->tokens[st][b]) = io->history[st * kBatch + b];
            __threadfence_system();
            *reinterpret_cast<volatile uint64_t *>(&p.stream->published) =
                (static_cast<uint64_t>(p.launch_id) << 32) | static_cast<uint32_t>(calls);
          }
        }
      }
      if (ok && kind != kQKV) ok = grid_barrier(p, s, ++barrier_index, 100 + ph);
    }
  }
  if (tid == 0) *s.prod_ctl = -1;   // producer: no more steps

  // 5. finish (:593-614) and emit (:296-324), CTA 0; a decoder step reports
  //    only its status and call count and leaves the resident state alone
  if (blockIdx.x == 0 && tid == 0 && step_mode) {
    io->control_out[3] = (!ok || aborted(p)) ? kModelError : w->status;
    io->control_out[4] = w->model_calls;
  } else if (blockIdx.x == 0 && tid == 0) {
    int32_t status = w->status;
    if (!ok || aborted(p)) status = kModelError;
    const bool good = status == kOk;
    for (int b = 0; b < kBatch; ++b) {
      if (!good) {
        w->reason[b] = kFallback;
      } else if (w->active0[b] == 1 && w->reason[b] == kNone) {
        w->reason[b] = kMaxStepsReason;
      }
    }
    if (good) {
      for (int b = 0; b < kBatch; ++b) {
        if (w->active0[b] == 0) continue;
        p.res->generation[b] = w->generation[b];
        p.res->token[b] = w->token[b];
        p.res->position[b] = w->position[b];
        p.res->length[b] = w->length[b];
        p.res->valid[b] = 1;
      }
    }
    int32_t *c = io->control_out;
    c[0] = w->max_steps;
    c[1] = w->sampling;
    c[2] = w->variant;
    c[3] = status;
    c[4] = w->model_calls;
    c[5] = w->importing ? static_cast<int32_t>(w->checksum) : (good ? 0 : 1);
    int init_count = 0, final_count = 0;
    for (int b = 0; b < kBatch; ++b) {
      c[6 + b] = w->eos[b];
      c[6 + kBatch + b] = w->active0[b];
      c[6 + 2 * kBatch + b] = w->executed[b];
      c[6 + 3 * kBatch + b] = w->reason[b];
      c[6 + 4 * kBatch + 2 + b] = w->active0[b] == 1 ? w->generation[b] : 0;
      init_count += w->active0[b] != 0;
      final_count += (good ? w->active[b] : w->active0[b]) != 0;
    }
    c[6 + 4 * kBatch] = init_count;
    c[6 + 4 * kBatch + 1] = final_count;
  }
}

}  // namespace cruise
