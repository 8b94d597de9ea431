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
// operand of 128 rows and 64 k values, without reshuffling.  The activations
// X (row-major bf16) arrive through a 2-D tensor map with the hardware's
// 128-byte swizzle.
//
// The kernel runs on CTA pairs (clusters of two, one CTA per SM) and the
// pair's MMAs are 2-SM tcgen05.mma (cta_group::2, M = 256): a pair tile is 256
// W rows x all T tokens (T <= 512, in halves of up to 256: one MMA each), over
// a range of k chunks (split-K where a projection has too few row tiles to
// fill the GPU).  Per k chunk each CTA holds its 128 W rows and its half of
// each token half (16 + 2 x 16 KB per stage; four stages), and its tensor
// memory holds its 128 rows x the tile's tokens (two accumulators of 256 fp32
// columns).  Every byte of W is read once per tile and every byte of X once
// per 256 rows: the tile is as large as the tensor memory allows, which
// matters more here than overlapping the epilogue with the next tile.  On
// the large projections the MMAs run close to the tensor pipe's rate at the
// clock the SMs hold under this load; a shallower ring (three stages) costs
// a few per cent, so the copies keep up.
//   warp 0         TMA producer (one thread per CTA): waits for its stage to
//                  be free, loads its W rows and tokens with the 2-SM form of
//                  the tensor copy, whose bytes complete on the leader CTA's
//                  stage barrier (the leader's producer arms it with both
//                  CTAs' bytes); it runs on into the next tile;
//   warp 1         TMEM allocation in both CTAs; in the leader CTA one thread
//                  issues the MMAs: per stage 4 k steps x the token halves of
//                  M = 256 x N = the half's tokens rounded up to 16; a
//                  multicast commit frees the stage in both CTAs and, after
//                  the tile's last chunk, tells both epilogues the
//                  accumulators are complete;
//   warps 2..17    epilogue (both CTAs): tcgen05.ld of their 32 TMEM lanes
//                  (W rows), 32 tokens at a time (four warps per lane quadrant
//                  take every fourth chunk of tokens), then either fp32
//                  partial sums [split][T][N] (the caller adds the splits in
//                  order, so the result is deterministic), staged 8 tokens x
//                  32 rows at a time in the warp's 2 KB of shared memory and
//                  written by tensor stores, or, for the
//                  interleaved gate/up projection, the SwiGLU of each (gate,
//                  up) row pair written as the bf16 activation [T][I] (the
//                  decoder's rounding points: bf16(silu(bf16 g)) * bf16 u,
//                  rounded once; silu from the fast exponential and
//                  division); for the SwiGLU the (g, u) pairs are read out
//                  first and the accumulators handed back to the leader's MMA
//                  thread before the arithmetic and the stores.
// Every wait is bounded (2 s): on expiry the CTA records an error and raises
// the abort flag in both CTAs, every role stops at its next wait, the pair
// lets the copies and MMAs in flight finish (bounded), meets at a cluster
// barrier, frees its tensor memory and returns.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cstdint>

#include "ptx.cuh"

namespace cruise {
namespace tcgemm {

constexpr int kEpilogueWarp0 = 2;          // warps 0 and 1: producer, MMA issuer
constexpr int kEpilogueWarps = 16;
constexpr int kEpilogueGroups = kEpilogueWarps / 4;   // epilogue warps per TMEM lane quadrant
constexpr int kThreads = 32 * (kEpilogueWarp0 + kEpilogueWarps);
constexpr int kM = 128;                    // W rows per CTA
constexpr int kRows = 2 * kM;              // W rows per pair tile (the MMA's M)
constexpr int kSub = 256;                  // tokens per MMA at most (its largest N): a token sub-tile
constexpr int kKChunk = 64;                // k values per stage (one 128-byte swizzle row)
constexpr uint32_t kWBytes = kM * kKChunk * 2;   // 16 KB: this CTA's W rows of a k chunk
constexpr uint32_t kRingBytes = 196608;    // the stage ring: 4 x 48 KB, 6 x 32 KB or 8 x 24 KB
constexpr int kMaxStages = 8;
constexpr uint32_t kAccCols = 256;         // one token sub-tile's accumulator: 256 fp32 columns
constexpr uint32_t kTmemCols = 512;        // two sub-tiles
constexpr uint64_t kTimeoutNs = 2000000000ull;
constexpr uint64_t kSettleNs = 50000ull;   // after a failure: time given to copies in flight

struct Args {
  int T;             // tokens (<= 512)
  int N;             // W rows
  int chunks;        // k chunks of 64 over the whole K
  int kc;            // the weight tiles' width (a multiple of 64)
  int nsplit;        // k ranges per (row tile, token tile)
  int mode;          // 0: fp32 partials, 1: SwiGLU of interleaved gate/up rows, 2: bf16 output
  int ttile;         // tokens per pair tile: 128, 256 or 512 (two sub-tiles of 256)
  int ttiles;        // token tiles: ceil(T / ttile)
  int tsub;          // token sub-tiles per tile (MMAs per k step): 1 or 2
  int xrows;         // tokens per CTA per sub-tile and k chunk: ttile / 2, at most 128 (the X box)
  int stages;        // ring depth: kRingBytes / stage bytes, at most kMaxStages
  int tiles;         // row tiles x token tiles x nsplit
  float *partials;   // mode 0: [nsplit][T][N]
  bf16 *out;         // mode 1: the activation [T][out_stride] (out_stride = N / 2); mode 2: [T][out_stride]
  int out_stride;
  uint32_t *error;   // set to the failing site when a wait ran out
  int w_evict_first; // W copies mark their L2 lines evict-first (W is read once; X and the partials stay)
  int p_evict_last;  // partial-sum stores mark their lines evict-last (the next kernel reads them)
  uint64_t *trace;   // profiling: [CTA][kTraceMarks] %globaltimer marks (null: off)
};

// Trace marks of one CTA: entry, predecessor complete, first load issued,
// first stage landed (leader), last MMA committed (leader), first
// accumulators ready (epilogue warp 2), epilogue warp 2 done, exit.
constexpr int kTraceMarks = 8;

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

// The same wait with cluster-scope acquire, for barriers the peer CTA arrives on.
__device__ __forceinline__ bool mbar_try_cluster(uint64_t *bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

__device__ __forceinline__ bool wait_phase_cluster(uint64_t *bar, uint32_t parity) {
  if (mbar_try_cluster(bar, parity)) return true;
  const uint64_t deadline = now_ns() + kTimeoutNs;
  while (true) {
    if (mbar_try_cluster(bar, parity)) return true;
    if (now_ns() > deadline) return false;
  }
}

__device__ __forceinline__ void mark(const Args &a, int i) {
  if (a.trace != nullptr) a.trace[blockIdx.x * kTraceMarks + i] = now_ns();
}

__device__ __forceinline__ void settle() {
  const uint64_t until = now_ns() + kSettleNs;
  while (now_ns() < until) __nanosleep(1000);
}

// ---- cluster ------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ uint32_t cluster_id() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}

__device__ __forceinline__ uint32_t cluster_count() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}

// The shared::cluster address of `local`'s counterpart in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t peer_addr(const void *local, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(smem_u32(local)), "r"(rank));
  return out;
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.aligned;\n\tbarrier.cluster.wait.aligned;" ::: "memory");
}

// One arrival on an mbarrier of another CTA of the cluster.
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

__device__ __forceinline__ void st_remote_u32(uint32_t cluster_addr, uint32_t v) {
  asm volatile("st.relaxed.cluster.shared::cluster.u32 [%0], %1;" ::"r"(cluster_addr), "r"(v) : "memory");
}

// ---- 2-SM tensor copies: this CTA's shared memory, the leader's barrier ----------
__device__ __forceinline__ void tma_load_5d_pair(void *dst, const CUtensorMap *map, int c0, int c1, int c2, int c3,
                                                 int c4, uint32_t bar_cluster) {
  asm volatile(
      "cp.async.bulk.tensor.5d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, "
      "%4, %5, %6}], [%7];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4), "r"(bar_cluster)
      : "memory");
}

// The same W copy with an L2 eviction-priority policy on its lines.
__device__ __forceinline__ void tma_load_5d_pair_hint(void *dst, const CUtensorMap *map, int c0, int c1, int c2,
                                                      int c3, int c4, uint32_t bar_cluster, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.5d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], "
      "[%1, {%2, %3, %4, %5, %6}], [%7], %8;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4), "r"(bar_cluster),
      "l"(policy)
      : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap *map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tma_load_2d_pair(void *dst, const CUtensorMap *map, int c0, int c1,
                                                 uint32_t bar_cluster) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, "
      "%3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(bar_cluster)
      : "memory");
}

// ---- tcgen05, 2-SM forms --------------------------------------------------------
// Allocation and deallocation are issued by the same warp in both CTAs of the pair.
__device__ __forceinline__ void tmem_alloc(uint32_t *dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
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
// fp32 accumulate, M = 256 (the pair), N = n (a multiple of 16, at most 256).
__host__ __device__ constexpr uint32_t idesc_m256(uint32_t n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((n >> 3) << 17) | ((256u >> 4) << 24);
}

// D (this CTA's TMEM and the peer's) [+]= A . B^T; A: this CTA's 128 rows at
// a_desc and the peer's 128 at the same offset; B: N / 2 rows here, N / 2 in the peer.
__device__ __forceinline__ void mma_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t accumulate,
                                         uint32_t idesc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %3, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %4, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(accumulate), "r"(idesc));
}

// One arrival on the barrier at this offset in both CTAs of the pair once
// every tcgen05 operation this thread issued before has completed.
__device__ __forceinline__ void commit_pair(uint64_t *bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(static_cast<uint16_t>(3))
      : "memory");
}

// The same, on this CTA's barrier only.
__device__ __forceinline__ void commit_local(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
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

// 16 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15])
               :
               : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  const __nv_bfloat162 p = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t *>(&p);
}

// Shared memory: the ring (1024-aligned), then the barriers and flags.
struct Bars {
  uint64_t full[kMaxStages];    // leader: a stage's bytes from both CTAs landed
  uint64_t empty[kMaxStages];   // both: the MMAs reading a stage completed
  uint64_t acc_full;         // both: the tile's MMAs completed
  uint64_t acc_empty;        // leader: both CTAs' epilogues read the accumulators out
  uint64_t drain;            // leader: all MMAs completed (exit path)
  uint32_t tmem_base;
  int abort;
};

// The SwiGLU epilogue keeps the (g, u) pairs of its last token slot here, the
// other three in registers: [word][epilogue thread].
constexpr int kStashWords = 16;
constexpr size_t kStashBytes = static_cast<size_t>(kStashWords) * kEpilogueWarps * 32 * 4;

// The barriers get a 1 KB slot after the ring, so the stash starts 1 KB
// aligned (the fp32 epilogue's tensor stores read it).
constexpr size_t kBarsSlot = 1024;
static_assert(sizeof(Bars) <= kBarsSlot, "barrier slot");
__host__ __device__ inline size_t smem_bytes() { return 1024 + kRingBytes + kBarsSlot + kStashBytes; }

// The fp32 epilogue stages 8 tokens x 32 W rows (1 KB) per tensor store, two
// such buffers per epilogue warp in its 2 KB of the stash.
constexpr int kStoreTokens = 8;

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Tensor store of a 32-row x 8-token fp32 box from shared memory into the
// partial sums [split][T][N] (coordinates: row, token, split; the parts of
// the box past N or T are not written).
__device__ __forceinline__ void tma_store_3d(const CUtensorMap *map, const void *src, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%1, %2, %3}], [%4];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(src))
               : "memory");
}

// The same store with an L2 eviction-priority policy on the written lines.
__device__ __forceinline__ void tma_store_3d_hint(const CUtensorMap *map, const void *src, int c0, int c1, int c2,
                                                  uint64_t policy) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group.L2::cache_hint [%0, {%1, %2, %3}], [%4], %5;" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(src)), "l"(policy)
               : "memory");
}

__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }

// At most one of this thread's bulk stores still reading shared memory.
__device__ __forceinline__ void bulk_wait_read1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }

// All of this thread's bulk stores complete (written to global memory).
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Shared-memory bytes of one stage per CTA: its W rows and its share of each sub-tile's tokens.
__host__ __device__ inline uint32_t stage_bytes(int tsub, int xrows) {
  return kWBytes + static_cast<uint32_t>(tsub * xrows * kKChunk * 2);
}

__device__ __forceinline__ float rbf16(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

// Tile t -> (row tile, token tile, split): 256 W rows x ttile tokens, chunks
// [c0, c1).  Neighbouring pairs take the token tiles of one row tile, so its
// W is fetched from HBM about once.
struct Tile {
  int mt, tq, split, c0, c1;
};

__device__ __forceinline__ Tile tile_of(const Args &a, int t) {
  Tile x;
  x.split = t % a.nsplit;
  const int r = t / a.nsplit;
  x.tq = r % a.ttiles;
  x.mt = r / a.ttiles;
  x.c0 = static_cast<int>(static_cast<int64_t>(a.chunks) * x.split / a.nsplit);
  x.c1 = static_cast<int>(static_cast<int64_t>(a.chunks) * (x.split + 1) / a.nsplit);
  return x;
}

// First token of sub-tile s of token tile tq, its token count (0 when it lies
// past T), and the MMA's N for it (rounded up to 16: each CTA holds N / 2).
__device__ __forceinline__ int sub_first(const Args &a, int tq, int s) { return tq * a.ttile + s * kSub; }

__device__ __forceinline__ int sub_tokens(const Args &a, int tq, int s) {
  const int left = a.T - sub_first(a, tq, s), most = a.ttile < kSub ? a.ttile : kSub;
  return left <= 0 ? 0 : left < most ? left : most;
}

__device__ __forceinline__ int sub_n(const Args &a, int tq, int s) { return (sub_tokens(a, tq, s) + 15) & ~15; }

// Records the failing site and raises the abort flag in both CTAs of the pair.
__device__ __forceinline__ void fail(const Args &a, Bars *b, uint32_t rank, uint32_t site) {
  atomicMax(a.error, site);
  *reinterpret_cast<volatile int *>(&b->abort) = 1;
  st_remote_u32(peer_addr(&b->abort, rank ^ 1u), 1u);
}

__device__ __forceinline__ bool aborted(Bars *b) { return *reinterpret_cast<volatile int *>(&b->abort) != 0; }

__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
                const __grid_constant__ CUtensorMap pmap, const Args a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *ring = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Bars *b = reinterpret_cast<Bars *>(ring + kRingBytes);
  uint32_t *stash = reinterpret_cast<uint32_t *>(ring + kRingBytes + kBarsSlot);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int pair = static_cast<int>(cluster_id()), npairs = static_cast<int>(cluster_count());
  const int S = a.stages;
  const uint32_t sbytes = stage_bytes(a.tsub, a.xrows), xbytes = static_cast<uint32_t>(a.xrows * kKChunk * 2);
  // launched as a dependent of the previous prefill kernel: let the next one
  // begin launching; the set-up below touches nothing the predecessor does
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (tid == 0) mark(a, 0);

  if (tid == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&b->full[i], 1);
      mbar_init(&b->empty[i], 1);
    }
    mbar_init(&b->acc_full, 1);
    mbar_init(&b->acc_empty, 2 * kEpilogueWarps);
    mbar_init(&b->drain, 1);
    b->abort = 0;
    mbar_fence_init();
  }
  if (warp == 1) {
    tmem_alloc(&b->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before_sync();
  // both CTAs' barriers are initialised before either CTA signals the other's
  cluster_sync();
  tc_fence_after_sync();
  const uint32_t tmem = b->tmem_base;
  // the predecessor's outputs (this GEMM's X) are complete and visible; the
  // producer thread waits inside its role, after its first W copies
  if (!(warp == 0 && lane == 0)) asm volatile("griddepcontrol.wait;" ::: "memory");
  if (tid == 32) mark(a, 1);

  if (warp == 0) {
    // ---- producer (both CTAs): chunk c is segment c % segs of k tile c / segs
    if (lane == 0) {
      const int segs = a.kc / kKChunk;
      const uint64_t policy = l2_policy_evict_first();
      prefetch_tensormap(&wmap);
      prefetch_tensormap(&xmap);
      int issued = 0;
      bool ok = true;
      auto load_w = [&](uint8_t *sa, int c, int mt, uint32_t bar) {
        // W: (element, segment, row in tile, k tile, row group); 8 row groups = this CTA's 128 rows
        const int rg = mt * (kRows / 16) + static_cast<int>(rank) * 8;
        if (a.w_evict_first)
          tma_load_5d_pair_hint(sa, &wmap, 0, c % segs, 0, c / segs, rg, bar, policy);
        else
          tma_load_5d_pair(sa, &wmap, 0, c % segs, 0, c / segs, rg, bar);
      };
      auto nsub_of = [&](const Tile &x) {
        int nsub = 0;   // sub-tiles with tokens
        for (int s = 0; s < a.tsub; ++s) nsub += sub_tokens(a, x.tq, s) > 0 ? 1 : 0;
        return nsub;
      };
      asm volatile("griddepcontrol.wait;" ::: "memory");
      for (int t = pair; ok && t < a.tiles; t += npairs) {
        const Tile x = tile_of(a, t);
        const int nsub = nsub_of(x);
        for (int c = x.c0; c < x.c1; ++c) {
          const int st = issued % S;
          const uint32_t round = static_cast<uint32_t>(issued / S);
          uint8_t *sa = ring + static_cast<size_t>(st) * sbytes;
          const uint32_t bar = peer_addr(&b->full[st], 0);
          if (aborted(b) || !wait_phase(&b->empty[st], (round & 1u) ^ 1u)) {
            if (!aborted(b)) fail(a, b, rank, 1u);
            ok = false;
            break;
          }
          if (leader) mbar_arrive_expect_tx(&b->full[st], 2 * (kWBytes + static_cast<uint32_t>(nsub) * xbytes));
          load_w(sa, c, x.mt, bar);
          // X: (k, token); of each sub-tile, this CTA's N / 2 tokens (rows past T read as zeros)
          for (int s = 0; s < nsub; ++s)
            tma_load_2d_pair(sa + kWBytes + s * xbytes, &xmap, c * kKChunk,
                             sub_first(a, x.tq, s) + static_cast<int>(rank) * (sub_n(a, x.tq, s) / 2), bar);
          if (issued == 0) mark(a, 2);
          ++issued;
        }
      }
      if (ok) {
        // the leader's last commits arrive on this CTA's stage barriers: wait
        // (bounded) for them before the CTA may leave
        for (int i = issued > S ? issued - S : 0; i < issued; ++i)
          if (!wait_phase(&b->empty[i % S], static_cast<uint32_t>(i / S) & 1u)) {
            if (!aborted(b)) fail(a, b, rank, 5u);
            break;
          }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---- MMA issuer (leader CTA): stage -> 4 k steps x the sub-tiles, M = 256, N = the sub-tile's tokens
    if (leader && lane == 0) {
      int used = 0, local = 0;
      bool ok = true;
      for (int t = pair; ok && t < a.tiles; t += npairs, ++local) {
        const Tile x = tile_of(a, t);
        const int n0 = sub_n(a, x.tq, 0), n1 = a.tsub > 1 ? sub_n(a, x.tq, 1) : 0;
        const uint32_t idesc0 = idesc_m256(static_cast<uint32_t>(n0 > 0 ? n0 : 16));
        const uint32_t idesc1 = idesc_m256(static_cast<uint32_t>(n1 > 0 ? n1 : 16));
        // the previous tile's accumulators have been read out by both epilogues
        if (local > 0 && (aborted(b) || !wait_phase_cluster(&b->acc_empty, static_cast<uint32_t>(local - 1) & 1u))) {
          if (!aborted(b)) fail(a, b, rank, 2u);
          break;
        }
        tc_fence_after_sync();
        for (int c = x.c0; c < x.c1; ++c) {
          const int st = used % S;
          const uint32_t round = static_cast<uint32_t>(used / S);
          if (aborted(b) || !wait_phase(&b->full[st], round & 1u)) {
            if (!aborted(b)) fail(a, b, rank, 3u);
            ok = false;
            break;
          }
          tc_fence_after_sync();
          if (used == 0) mark(a, 3);
          const uint32_t sw = smem_u32(ring + static_cast<size_t>(st) * sbytes);
#pragma unroll
          for (int j = 0; j < kKChunk / 16; ++j) {
            const uint64_t ad = desc_sw128(sw + j * 32);
            const uint32_t acc = (c > x.c0 || j > 0) ? 1u : 0u;
            if (n0 > 0) mma_pair(tmem, ad, desc_sw128(sw + kWBytes + j * 32), acc, idesc0);
            if (n1 > 0) mma_pair(tmem + kAccCols, ad, desc_sw128(sw + kWBytes + xbytes + j * 32), acc, idesc1);
          }
          commit_pair(&b->empty[st]);
          ++used;
        }
        if (!ok) break;
        commit_pair(&b->acc_full);   // with no k chunks: completes at once, the epilogue writes zeros
      }
      mark(a, 4);
      // every MMA this thread issued has completed once `drain` fires
      commit_local(&b->drain);
      wait_phase(&b->drain, 0);
    }
    __syncwarp();
  } else {
    // ---- epilogue (both CTAs): warp w reads TMEM lanes 32 (w % 4) .. + 31
    // (its W rows) for the token chunks 32 g + 128 j of each sub-tile, g = its group
    const int quad = warp & 3, group = (warp - kEpilogueWarp0) >> 2;
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(quad * 32) << 16);
    const uint32_t leader_empty = peer_addr(&b->acc_empty, 0);
    int local = 0;
    for (int t = pair; t < a.tiles; t += npairs, ++local) {
      const Tile x = tile_of(a, t);
      bool ok = !aborted(b) && wait_phase(&b->acc_full, static_cast<uint32_t>(local) & 1u);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) {
        if (lane == 0 && !aborted(b)) fail(a, b, rank, 4u);
        break;
      }
      tc_fence_after_sync();
      if (local == 0 && warp == kEpilogueWarp0 && lane == 0) mark(a, 5);
      const bool zero = x.c1 <= x.c0;
      const int row = x.mt * kRows + static_cast<int>(rank) * kM + quad * 32 + lane;   // this thread's W row
      if (a.mode == 0) {
        // fp32 partial sums through tensor stores: the warp writes 8 tokens
        // of its 32 rows into one of its two 1 KB stash buffers, lane 0
        // stores the box; the other buffer's store may still be reading
        float *slice = reinterpret_cast<float *>(stash) + (warp - kEpilogueWarp0) * (2 * kStoreTokens * 32);
        const int row0 = x.mt * kRows + static_cast<int>(rank) * kM + quad * 32;
        const uint64_t keep = l2_policy_evict_last();
        int stores = 0;
        for (int s = 0; s < a.tsub; ++s) {
          const int ntok = sub_tokens(a, x.tq, s), first = sub_first(a, x.tq, s);
          const uint32_t acc = lane_addr + static_cast<uint32_t>(s) * kAccCols;
          for (int t0 = 32 * group; t0 < ntok; t0 += 32 * kEpilogueGroups) {
            float v[32];
            if (!zero) {
              tmem_ld32(acc + static_cast<uint32_t>(t0), v);
            } else {
#pragma unroll
              for (int q = 0; q < 32; ++q) v[q] = 0.f;
            }
#pragma unroll
            for (int h = 0; h < 32 / kStoreTokens; ++h) {
              if (t0 + h * kStoreTokens < ntok) {
                float *buf = slice + (stores & 1) * (kStoreTokens * 32);
                if (lane == 0 && stores >= 2) bulk_wait_read1();
                __syncwarp();
#pragma unroll
                for (int q = 0; q < kStoreTokens; ++q) buf[q * 32 + lane] = v[h * kStoreTokens + q];
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {   // boxes reaching past N or T are clipped; one wholly past N is skipped
                  if (row0 < a.N) {
                    if (a.p_evict_last)
                      tma_store_3d_hint(&pmap, buf, row0, first + t0 + h * kStoreTokens, x.split, keep);
                    else
                      tma_store_3d(&pmap, buf, row0, first + t0 + h * kStoreTokens, x.split);
                  }
                  bulk_commit();
                }
                ++stores;
              }
            }
          }
        }
        // the stores are complete before the kernel (and the caller's next
        // kernel) can end; the stash buffers are free for the next tile
        if (lane == 0) bulk_wait_all();
        tc_fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(leader_empty);
      } else if (a.mode == 2) {
        for (int s = 0; s < a.tsub; ++s) {
          const int ntok = sub_tokens(a, x.tq, s), first = sub_first(a, x.tq, s);
          const uint32_t acc = lane_addr + static_cast<uint32_t>(s) * kAccCols;
          for (int t0 = 32 * group; t0 < ntok; t0 += 32 * kEpilogueGroups) {
            float v[32];
            if (!zero) {
              tmem_ld32(acc + static_cast<uint32_t>(t0), v);
            } else {
#pragma unroll
              for (int q = 0; q < 32; ++q) v[q] = 0.f;
            }
            if (row < a.N) {
              bf16 *dst = a.out + static_cast<int64_t>(first + t0) * a.out_stride + row;
#pragma unroll
              for (int q = 0; q < 32; ++q)
                if (t0 + q < ntok) dst[static_cast<int64_t>(q) * a.out_stride] = __float2bfloat16_rn(v[q]);
            }
          }
        }
        // this CTA's rows of the accumulators are free for the pair's next tile
        tc_fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(leader_empty);
      } else {
        // rows 16g .. 16g+7 are gate rows, 16g+8 .. 16g+15 the matching up
        // rows: a gate lane and its up lane (8 lanes on) hold a pair for every
        // token.  The gate lane takes the even tokens, the up lane the odd
        // ones, each sending the other the half of the pair it needs.  The
        // pairs are read out of tensor memory first, rounded to bf16 (as the
        // SwiGLU takes them) and kept packed in registers, so the accumulators
        // go back to the MMA thread before the SwiGLU and the stores.
        // Slot 2 s + j: token chunk 32 group + 128 j of sub-tile s; slot 3
        // lives in shared memory (the registers hold three).
        const bool gate_lane = (lane & 15) < 8;
        const int odd = gate_lane ? 0 : 1;
        const int et = tid - 32 * kEpilogueWarp0;   // epilogue thread
        uint32_t gu[3][16];   // per slot: (g, u) of the lane's 16 tokens
#pragma unroll
        for (int sl = 0; sl < 4; ++sl) {
          const int s = sl >> 1, t0 = 32 * group + 128 * (sl & 1);
          if (s < a.tsub && t0 < sub_tokens(a, x.tq, s)) {
#pragma unroll
            for (int p = 0; p < 2; ++p) {   // two loads of 16 columns
              float v[16];
              if (!zero) {
                tmem_ld16(lane_addr + static_cast<uint32_t>(s * kAccCols + t0 + 16 * p), v);
              } else {
#pragma unroll
                for (int q = 0; q < 16; ++q) v[q] = 0.f;
              }
#pragma unroll
              for (int q = 0; q < 16; q += 2) {
                const float up_even = __shfl_down_sync(0xffffffffu, v[q], 8);      // gate lane <- u(q)
                const float gate_odd = __shfl_up_sync(0xffffffffu, v[q + 1], 8);   // up lane <- g(q + 1)
                const uint32_t w = pack_bf16(gate_lane ? v[q] : gate_odd, gate_lane ? up_even : v[q + 1]);
                if (sl < 3)
                  gu[sl < 3 ? sl : 0][8 * p + q / 2] = w;
                else
                  stash[(8 * p + q / 2) * (kEpilogueWarps * 32) + et] = w;
              }
            }
          }
        }
        tc_fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(leader_empty);
        const int i = (row >> 4) * 8 + (row & 7);   // intermediate index of the pair
#pragma unroll 1
        for (int sl = 0; sl < 4; ++sl) {
          const int s = sl >> 1, t0 = 32 * group + 128 * (sl & 1);
          const int ntok = s < a.tsub ? sub_tokens(a, x.tq, s) : 0;
          if (t0 < ntok && row < a.N) {
            uint32_t cur[16];
#pragma unroll
            for (int k = 0; k < 16; ++k)
              cur[k] = sl == 0 ? gu[0][k] : sl == 1 ? gu[1][k] : sl == 2 ? gu[2][k] : stash[k * (kEpilogueWarps * 32) + et];
            bf16 *dst = a.out + static_cast<int64_t>(sub_first(a, x.tq, s) + t0 + odd) * a.out_stride + i;
#pragma unroll
            for (int k = 0; k < 16; ++k) {
              if (t0 + 2 * k + odd < ntok) {
                const __nv_bfloat162 p = *reinterpret_cast<const __nv_bfloat162 *>(&cur[k]);
                const float g = __low2float(p), u = __high2float(p);
                // silu(g) = g / (1 + e^-g) with the fast exponential and
                // division (a few fp32 ulps, then rounded to bf16 as the
                // decoder rounds it)
                const float silu = rbf16(__fdividef(g, __fadd_rn(1.0f, __expf(-g))));
                dst[static_cast<int64_t>(2 * k) * a.out_stride] = __float2bfloat16_rn(__fmul_rn(silu, u));
              }
            }
          }
        }
      }
    }
  }
  if (warp == kEpilogueWarp0 && lane == 0) mark(a, 6);
  // after a failure, copies and commits still in flight get time to land
  // before the pair meets for the last time and frees its tensor memory
  if (aborted(b)) settle();
  tc_fence_before_sync();
  cluster_sync();
  tc_fence_after_sync();
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
  if (tid == 0) mark(a, 7);
}

}  // namespace tcgemm
}  // namespace cruise
