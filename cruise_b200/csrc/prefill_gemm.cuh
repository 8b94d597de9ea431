// prefill_gemm.cuh -- the batched prefill's projections on the 5th-generation
// tensor cores (sm_100a): Y[T][N] = X[T][K] . W[N][K]^T with the weights read
// straight from the engine's tiled decode layout (no second copy of them).
//
// The engine stores a projection as tiles of 16 rows x kc columns, each row's
// 16-byte units permuted unit ^ (row & 7).  Every 128-byte segment (64 k
// values) of such a row is therefore already in the 128-byte-swizzled order
// the tensor cores read for row (row & 7).  A five-dimensional TMA tensor map
// over that layout -- (64 elements, segment, row in tile, k tile, row group)
// -- gathers 8 row groups x 16 rows of one segment into 128 consecutive
// 128-byte rows of shared memory: exactly a K-major, 128-byte-swizzled
// operand of 128 rows (M = 128) and 64 k values, without reshuffling.  The
// activations X (row-major bf16) arrive through a 2-D tensor map with the
// hardware's 128-byte swizzle, 256 tokens per box (N = 256 per MMA).
//
// A persistent CTA of 576 threads walks tiles of 256 W rows x one 256-token
// half of X (T <= 512) over a range of k chunks (split-K where a projection
// has too few row tiles to fill the GPU).  The two 128-row halves of the tile
// are two M = 128 accumulators of up to 256 fp32 columns each -- all 512 TMEM
// columns -- fed by the same X tile, so each X byte brought into shared
// memory serves two MMAs and each W byte is brought in once per tile:
//   warp 0         TMA producer (one thread): a ring of 3 stages, each one
//                  k chunk of W (32 KB) and of X (32 KB), completed on
//                  mbarriers with the byte count; it runs on into the next
//                  tile while the epilogue drains the last one;
//   warp 1         MMA issuer (one thread): per stage 4 k steps x 2 row halves
//                  of tcgen05.mma.kind::f16 (N = the half's tokens rounded up
//                  to 16); tcgen05.commit frees the stage, and after the last
//                  chunk signals the epilogue; the next tile's MMAs wait until
//                  the epilogue has read the accumulators out;
//   warps 2..17    epilogue: tcgen05.ld of their 32 TMEM lanes (W rows), 32
//                  tokens at a time (four warps per lane quadrant take every
//                  fourth chunk of tokens), then either fp32 partial sums
//                  [split][T][N] (the caller adds the splits in order, so the
//                  result is deterministic) or, for the interleaved gate/up
//                  projection, the SwiGLU of each (gate, up) row pair written
//                  as the bf16 activation [T][I] (the decoder's rounding
//                  points: bf16(silu(bf16 g)) * bf16 u, rounded once).
// Every wait is bounded: on expiry the CTA records an error, every role stops
// at its next wait, the copies and MMAs in flight are waited for (bounded),
// the tensor memory is freed and the CTA returns.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cstdint>

#include "ptx.cuh"

namespace cruise {
namespace tcgemm {

constexpr int kThreads = 576;              // producer warp, MMA warp, 16 epilogue warps
constexpr int kEpilogueWarp0 = 2;          // first epilogue warp
constexpr int kEpilogueGroups = 4;         // epilogue warps per TMEM lane quadrant
constexpr int kM = 128;                    // W rows per MMA (M)
constexpr int kRows = 2 * kM;              // W rows per tile: two accumulators
constexpr int kTokHalf = 256;              // tokens per tile (the MMA's largest N)
constexpr int kKChunk = 64;                // k values per stage (one 128-byte swizzle row)
constexpr uint32_t kWBytes = kRows * kKChunk * 2;       // 32 KB
constexpr uint32_t kXBytes = kTokHalf * kKChunk * 2;    // 32 KB
constexpr uint32_t kStageBytes = kWBytes + kXBytes;
constexpr int kMaxStages = 3;
constexpr uint64_t kTimeoutNs = 2000000000ull;

struct Args {
  int T;             // tokens (<= 512)
  int N;             // W rows
  int chunks;        // k chunks of 64 over the whole K
  int kc;            // the weight tiles' width (a multiple of 64)
  int nsplit;        // k ranges per (row tile, token half)
  int mode;          // 0: fp32 partials, 1: SwiGLU of interleaved gate/up rows
  int stages;        // ring depth (<= kMaxStages)
  int halves;        // token halves (1 or 2)
  int tiles;         // row tiles x halves x nsplit
  float *partials;   // mode 0: [nsplit][T][N]
  bf16 *act;         // mode 1: [T][act_stride]
  int act_stride;    // mode 1: intermediate size I (N = 2 I)
  uint32_t *error;   // set to the failing site when a wait ran out
};

__device__ __forceinline__ uint64_t now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded mbarrier wait (true: phase `parity` completed).
__device__ __forceinline__ bool wait_phase(uint64_t *bar, uint32_t parity) {
  if (mbar_try(bar, parity)) return true;
  const uint64_t deadline = now_ns() + kTimeoutNs;
  while (true) {
    if (mbar_try(bar, parity)) return true;
    if (now_ns() > deadline) return false;
  }
}

__device__ __forceinline__ void tma_load_5d(void *dst, const CUtensorMap *map, int c0, int c1, int c2, int c3,
                                            int c4, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5, "
      "%6}], [%7];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int c0, int c1, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}

// ---- tcgen05 -----------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t *dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before_sync() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tc_fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory descriptor of a K-major operand in the canonical 128-byte
// swizzled layout: 128-byte rows, 8-row atoms of 1024 bytes (stride byte
// offset 1024), atoms 1024-byte aligned; `addr` may carry a k offset of 32
// bytes per 16-element step inside the row.
__device__ __forceinline__ uint64_t desc_sw128(uint32_t addr) {
  return static_cast<uint64_t>((addr >> 4) & 0x3FFFu) | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}

// Instruction descriptor of tcgen05.mma kind::f16: bf16 A and B (K-major),
// fp32 accumulate, M = 128, N = n (a multiple of 16, at most 256).
__host__ __device__ constexpr uint32_t idesc_m128(uint32_t n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((n >> 3) << 17) | ((128u >> 4) << 24);
}

__device__ __forceinline__ void mma(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t accumulate,
                                    uint32_t idesc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %3, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %4, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(accumulate), "r"(idesc));
}

// The mbarrier receives one arrival once every tcgen05 operation this thread
// issued before has completed.
__device__ __forceinline__ void commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 32 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                 "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                 "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__host__ __device__ inline size_t smem_bytes(int stages) {
  // 1 KB of slack to align the ring to 1024 bytes, the ring, then barriers
  return 1024 + static_cast<size_t>(stages) * kStageBytes + (2 * kMaxStages + 4) * 8 + 16;
}

__device__ __forceinline__ float rbf16(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

// Tile t -> (row tile, token half, split); neighbouring CTAs take the two
// halves of one row tile, so its W is fetched from HBM about once.
struct Tile {
  int mt, half, split, c0, c1, ntok;
};

__device__ __forceinline__ Tile tile_of(const Args &a, int t) {
  Tile x;
  x.split = t % a.nsplit;
  const int mh = t / a.nsplit;
  x.half = mh % a.halves;
  x.mt = mh / a.halves;
  x.c0 = static_cast<int>(static_cast<int64_t>(a.chunks) * x.split / a.nsplit);
  x.c1 = static_cast<int>(static_cast<int64_t>(a.chunks) * (x.split + 1) / a.nsplit);
  const int left = a.T - x.half * kTokHalf;
  x.ntok = left < kTokHalf ? left : kTokHalf;
  return x;
}

__device__ __forceinline__ void fail(const Args &a, volatile int *abort_flag, uint32_t site) {
  atomicMax(a.error, site);
  *abort_flag = 1;
}

__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap, const Args a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = a.stages;
  uint64_t *full = reinterpret_cast<uint64_t *>(base + static_cast<size_t>(S) * kStageBytes);
  uint64_t *empty = full + kMaxStages;
  uint64_t *acc_full = empty + kMaxStages;   // MMAs of a tile done
  uint64_t *acc_empty = acc_full + 1;        // epilogue read the accumulators out
  uint64_t *drain = acc_empty + 1;           // MMA thread: all its MMAs done (exit path)
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  constexpr uint32_t kTmemCols = 512;

  if (tid == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, kThreads / 32 - kEpilogueWarp0);
    mbar_init(drain, 1);
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---- producer: chunk c covers k = 64c .. 64c + 63, i.e. segment c % segs of k tile c / segs
    int issued = 0;
    if (lane == 0) {
      const int segs = a.kc / kKChunk;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < a.tiles; t += gridDim.x) {
        const Tile x = tile_of(a, t);
        for (int c = x.c0; c < x.c1; ++c) {
          const int st = issued % S;
          const uint32_t round = static_cast<uint32_t>(issued / S);
          if (*abort_flag || !wait_phase(&empty[st], (round & 1u) ^ 1u)) {
            if (!*abort_flag) fail(a, abort_flag, 1u);
            ok = false;
            break;
          }
          uint8_t *sa = base + static_cast<size_t>(st) * kStageBytes;
          mbar_arrive_expect_tx(&full[st], kStageBytes);
          // W: (element, segment, row in tile, k tile, row group); 16 row groups = 256 rows
          tma_load_5d(sa, &wmap, 0, c % segs, 0, c / segs, x.mt * (kRows / 16), &full[st]);
          // X: (k, token); rows past T read as zeros
          tma_load_2d(sa + kWBytes, &xmap, c * kKChunk, x.half * kTokHalf, &full[st]);
          ++issued;
        }
      }
      // copies still landing (after a failure anywhere in the CTA) must not
      // outlive it: wait (bounded) for the last ring's worth
      for (int i = issued > S ? issued - S : 0; i < issued; ++i)
        wait_phase(&full[i % S], static_cast<uint32_t>(i / S) & 1u);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---- MMA issuer: stage -> 4 k steps x 2 row halves into accumulators at columns 0 and 256
    if (lane == 0) {
      int used = 0, local = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < a.tiles; t += gridDim.x, ++local) {
        const Tile x = tile_of(a, t);
        const uint32_t idesc = idesc_m128(static_cast<uint32_t>((x.ntok + 15) & ~15));
        if (local > 0 && (*abort_flag || !wait_phase(acc_empty, static_cast<uint32_t>(local - 1) & 1u))) {
          if (!*abort_flag) fail(a, abort_flag, 2u);
          break;
        }
        tc_fence_after_sync();
        for (int c = x.c0; c < x.c1; ++c) {
          const int st = used % S;
          const uint32_t round = static_cast<uint32_t>(used / S);
          if (*abort_flag || !wait_phase(&full[st], round & 1u)) {
            if (!*abort_flag) fail(a, abort_flag, 3u);
            ok = false;
            break;
          }
          tc_fence_after_sync();
          const uint32_t sw = smem_u32(base + static_cast<size_t>(st) * kStageBytes);
          const uint32_t sx = sw + kWBytes;
#pragma unroll
          for (int j = 0; j < kKChunk / 16; ++j) {
            const uint32_t acc = (c > x.c0 || j > 0) ? 1u : 0u;   // the tile's first k step overwrites
            const uint64_t bd = desc_sw128(sx + j * 32);
            mma(tmem, desc_sw128(sw + j * 32), bd, acc, idesc);
            mma(tmem + kTokHalf, desc_sw128(sw + kM * 128 + j * 32), bd, acc, idesc);
          }
          commit(&empty[st]);
          ++used;
        }
        if (!ok) break;
        if (x.c1 > x.c0)
          commit(acc_full);
        else
          mbar_arrive(acc_full);   // no k chunks: the epilogue writes zeros
      }
      // every MMA this thread issued has completed once `drain` fires
      commit(drain);
      wait_phase(drain, 0);
    }
    __syncwarp();
  } else {
    // ---- epilogue: warp w reads TMEM lanes 32 (w % 4) .. + 31 (its W rows of
    // both accumulators) for the token chunks 32 g + 128 j, g = its group
    const int quad = warp & 3, group = (warp - kEpilogueWarp0) >> 2;
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    int local = 0;
    for (int t = blockIdx.x; t < a.tiles; t += gridDim.x, ++local) {
      const Tile x = tile_of(a, t);
      bool ok = !*abort_flag && wait_phase(acc_full, static_cast<uint32_t>(local) & 1u);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) {
        if (lane == 0 && !*abort_flag) fail(a, abort_flag, 4u);
        break;
      }
      tc_fence_after_sync();
      const bool zero = x.c1 <= x.c0;
      for (int h = 0; h < 2; ++h) {
        const int row = x.mt * kRows + h * kM + quad * 32 + lane;   // this thread's W row
        for (int t0 = 32 * group; t0 < x.ntok; t0 += 32 * kEpilogueGroups) {
          float v[32];
          if (!zero) {
            tmem_ld32(lane_addr + static_cast<uint32_t>(h * kTokHalf + t0), v);
          } else {
#pragma unroll
            for (int q = 0; q < 32; ++q) v[q] = 0.f;
          }
          const int tok0 = x.half * kTokHalf + t0;
          if (a.mode == 0) {
            if (row < a.N) {
              float *dst = a.partials + (static_cast<int64_t>(x.split) * a.T + tok0) * a.N + row;
#pragma unroll
              for (int q = 0; q < 32; ++q)
                if (t0 + q < x.ntok) dst[static_cast<int64_t>(q) * a.N] = v[q];
            }
          } else {
            // rows 16g .. 16g+7 are gate rows, 16g+8 .. 16g+15 the matching up rows
            const bool gate_lane = (lane & 15) < 8;
            const int i = (row >> 4) * 8 + (row & 7);   // intermediate index of the pair
            bf16 *dst = a.act + static_cast<int64_t>(tok0) * a.act_stride + i;
#pragma unroll
            for (int q = 0; q < 32; ++q) {
              const float up = __shfl_down_sync(0xffffffffu, v[q], 8);
              if (gate_lane && row < a.N && t0 + q < x.ntok) {
                const float g = rbf16(v[q]), u = rbf16(up);
                const float silu = rbf16(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))));
                dst[static_cast<int64_t>(q) * a.act_stride] = __float2bfloat16_rn(__fmul_rn(silu, u));
              }
            }
          }
        }
      }
      // the accumulators are free for the next tile's MMAs
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(acc_empty);
    }
  }
  tc_fence_before_sync();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, kTmemCols);
}

}  // namespace tcgemm
}  // namespace cruise
