// epoch_types.h -- device data layout of the resident decode epoch, shared by
// the host engine (engine.cu) and the persistent epoch kernel (epoch_kernel.cuh).
#pragma once

#include <cstdint>
#include <cuda_bf16.h>

namespace cruise {

using bf16 = __nv_bfloat16;

constexpr int kBatch = 4;             // static rows per epoch (controller :16)
constexpr int kMaxSteps = 8;          // max K (controller :17)
constexpr int kMaxBlocksPerRow = 8;   // capacity of the block-table buffers
constexpr int kControlIn = 11;        // [K, eos x4, sampling, variant, gen x4]
constexpr int kControlOut = 28;       // emit layout (controller :296-324)
constexpr int kTilingBytes = 72;
constexpr int kImportFlag = 0x100;

constexpr int kRows = 16;             // weight rows per tile (one m16 MMA slab)
constexpr int kMaxKc = 512;           // k elements per tile (power of two, 64..512)
constexpr int kStageBytes = 32768;    // one bulk copy: consecutive tiles of the stream
constexpr int kConsumerWarps = 8;
constexpr int kConsumerThreads = kConsumerWarps * 32;
constexpr int kProducerWarp = kConsumerWarps;          // warp 8: weight producer (TMA)
constexpr int kEpilogueWarp = kConsumerWarps + 1;      // warp 9: reductions and epilogues
constexpr int kThreads = kConsumerThreads + 64;
constexpr int kRedSlots = 4;                           // row-group partial-sum ring
constexpr int kMaxCtas = 1024;
constexpr int kMaxStages = 8;
constexpr int kTraceMax = 2048;       // grid barriers recorded per launch
constexpr int kTraceSeries = 6;      // globaltimer series per grid barrier (see cruise_epoch_read_trace)
constexpr int kTraceCtaWords = 12;    // per-CTA marks per grid barrier (see cruise_epoch_read_trace_cta)

// statuses and finish reasons of the reference controller (:51-74)
enum Status : int32_t {
  kOk = 0,
  kInvalidMetadata = 201,
  kCapacityExceeded = 202,
  kInvalidBlockTable = 203,
  kSlotMismatch = 204,
  kUnsupportedSampling = 205,
  kUnsupportedGraph = 206,
  kModelError = 207,
  kInvalidModelOutput = 208,
  kNonFiniteLogits = 209,
  kPositionProgress = 210,
  kAllocationFailure = 211,
  kResidentContinuity = 212,
};
enum Finish : int32_t { kNone = 0, kEos = 1, kMaxStepsReason = 2, kFallback = 3, kEmpty = 4, kAlreadyFinished = 5 };

// What one launch runs: a resident epoch (the controller and up to K decoder
// steps), or one decoder step of the 9-in / 4-out decoder ABI (logits and the
// next positions out, K/V updated in place, no controller and no resident state).
enum LaunchMode : int32_t { kModeEpoch = 0, kModeDecoderStep = 1 };

// Per-rank geometry.  Without tensor parallelism the rank holds the whole
// model; with it (tp ranks) the rank holds query heads [q0, q0 + nq), KV heads
// [kv0, kv0 + nkv) of nkv_all, intermediate rows [i0, i0 + I) and vocabulary
// rows [v0, v0 + Vl); the residual stream (H) and the embedding are whole.
struct ModelDims {
  int32_t L, H, nq, nkv, d, I, I_pad, V, V_pad, Nqkv;
  int32_t Hq;            // attention output width on this rank (nq * d)
  int32_t Kq;            // the O projection's input columns: Hq, zero-padded (see fill_dims)
  int32_t Vl;            // lm_head rows on this rank (V without tensor parallelism)
  int32_t v0;            // global id of this rank's first vocabulary row
  int32_t kv0, nkv_all;  // first KV head of this rank, KV heads of the model
  int32_t q0;            // first query head of this rank
  float eps;
  float sqrt_d;          // (float)sqrt(head_dim), the attention divisor
  int32_t bs, bpr, NB, C;
};

// Projection matrices are stored TILED: tile (rg, kk) holds rows rg*16..+15,
// columns kk*kc..+kc-1 as 16 contiguous rows of kc bf16 with the 16-byte units
// of row r permuted by unit ^ (r & 7) (conflict-free 128-bit shared loads);
// tiles are laid out in stream order [rg][kk], so any run of consecutive tiles
// is one contiguous block of HBM.  Logical shapes:
struct LayerWeights {
  const bf16 *w_in, *w_post;   // [H]
  const bf16 *qkv_w;           // tiled [Nqkv][H]   rows: q | k | v
  const bf16 *qkv_b;           // [Nqkv]
  const bf16 *o_w;             // tiled [H][Kq]: columns >= Hq are zero
  const bf16 *gu_w;            // tiled [2I][H]: per 16 rows, 8 gate rows then the 8 matching up rows
  const bf16 *down_w;          // tiled [H][I_pad]  columns >= I are zero
};

// Streaming egress, in host-mapped pinned memory: after each decode step of an
// epoch the kernel writes that step's tokens (-1 for rows that did not run),
// then `published` = launch id << 32 | steps so far.
struct StreamRing {
  int64_t tokens[kMaxSteps][kBatch];
  uint64_t published;
};

// One host->device and one device->host copy per epoch (the 8-in / 2-out ABI).
struct EpochIO {
  int64_t token[kBatch];
  int64_t position[kBatch];
  int32_t seq_len[kBatch];
  int32_t slot[kBatch];
  int32_t active[kBatch];
  int32_t block_table[kBatch * kMaxBlocksPerRow];
  int32_t control[kControlIn];
  uint8_t tiling[kTilingBytes];
  int32_t use_forced;                    // 1: forced[] overrides argmax (device prefill)
  int64_t forced[kMaxSteps * kBatch];    // [step][row] teacher-forced next token, -1 = greedy
  // outputs
  int64_t history[kMaxSteps * kBatch];   // [step][row]
  int32_t control_out[kControlOut];
};

// Per-row resident state kept across epochs (controller :624-631).
struct ResidentState {
  int32_t generation[kBatch];
  int32_t valid[kBatch];
  int32_t length[kBatch];
  int32_t pad0[kBatch];
  int64_t token[kBatch];
  int64_t position[kBatch];
};

// Working state of the running epoch (written by CTA 0, read by all).
struct EpochWork {
  int64_t token[kBatch];
  int64_t position[kBatch];
  int32_t length[kBatch];
  int32_t slot[kBatch];
  int32_t active[kBatch];
  int32_t active0[kBatch];
  int32_t executed[kBatch];
  int32_t reason[kBatch];
  int32_t new_gen[kBatch];
  int32_t eos[kBatch];
  int32_t generation[kBatch];
  int32_t bt[kBatch * kMaxBlocksPerRow];
  int32_t status;
  int32_t model_calls;
  int32_t stop;          // 1: leave the step loop
  int32_t importing;
  int32_t import_rows;   // rows whose payload is copied
  int32_t max_steps;
  int32_t sampling;
  int32_t variant;
  uint32_t checksum;
  int32_t pad0;
  uint64_t adler[2 * 64 * kBatch * 2];  // per imported block: (S1, S2)
};

// Cross-CTA synchronisation words; zeroed by the host before every launch,
// together with the grid's tagged partial-sum words that follow it.
constexpr int kBarrierLanes = 8;     // arrival counters of the grid barrier
constexpr int kMaxKvGroups = 16;     // KV heads per rank with their own QKV completion counter
struct SyncState {
  uint32_t barrier[kBarrierLanes][32];   // CTA c arrives on counter c % 8 (one 128-B line each)
  uint32_t error;              // non-zero: a wait timed out, every CTA leaves
  uint32_t error_where;
  uint32_t pad0[30];
  // QKV row groups finished per KV head (one 128-B line each), over the whole
  // launch: attention units of a KV head start once its count reaches
  // (row groups of the head) x (QKV phases so far); no grid barrier between
  uint32_t qkv_done[kMaxKvGroups][32];
};
// Bytes the host clears before a launch: SyncState, then [grid][64] tagged
// split row-group partial sums (fp32 value | phase sequence number << 32).
__host__ __device__ inline size_t sync_bytes(int grid) {
  return sizeof(SyncState) + static_cast<size_t>(grid) * 64 * sizeof(uint64_t);
}

// One rank's block of the tensor-parallel exchange, written by its peers over
// NVLink: the fp32 row-parallel partials of the O and down projections
// (double-buffered: set 0 for O, set 1 for down) from every rank, the lm_head
// argmax partials from every rank, and one sequence flag per source rank.
constexpr int kMaxTp = 8;
struct TpArg {
  float val;
  int32_t idx, bad, pad;
};
constexpr int kTpRows = 8192;          // widest hidden size a tensor-parallel exchange holds

struct TpExchange {
  uint32_t flag[kMaxTp][32];            // flag[src]: last argmax-exchange sequence number src published (own 128-B line)
  TpArg arg[kMaxTp][4];                 // argmax partial of each rank per batch row
  // [set][src][n][b]: rank src's fp32 partial of output row n, batch row b, in
  // the low half of the word and the sequence number of its phase in the high
  // half (H <= kTpRows); set 0 holds the O projection, set 1 the down projection
  uint64_t part[2][kMaxTp][kTpRows][4];
};

struct EpochParams {
  ModelDims m;
  const LayerWeights *layers;  // [L] in device memory
  const bf16 *embed;           // [V][H]
  const bf16 *final_norm;      // [H]
  const bf16 *lm_head;         // [V_pad][H]
  const bf16 *rope_cos;        // [C][d]
  const bf16 *rope_sin;        // [C][d]
  bf16 *key_cache;             // [L][NB][bs][nkv][d]
  bf16 *value_cache;
  bf16 *h;                     // [4][H] residual stream
  bf16 *qkv;                   // [4][Nqkv]
  bf16 *attn;                  // [4][H]
  bf16 *act;                   // [4][I_pad]
  uint64_t *partials;          // [G][64] split row-group partial sums as tagged words (after SyncState)
  float *arg_val;              // [G][4]
  int32_t *arg_idx;            // [G][4]
  int32_t *arg_bad;            // [G][4]
  float *logits;               // optional [8][4][V]
  const uint8_t *import_payload;  // device copy of the import payload
  EpochIO *io;
  ResidentState *res;
  EpochWork *work;
  SyncState *sync;
  int32_t grid;                // CTAs (one per SM)
  int32_t stages;              // weight ring depth
  int32_t xs_stride;           // activation row stride in smem (elements)
  int32_t down_xglobal;        // 1: the down projection reads its input from L2, not smem
  int32_t o_xglobal;           // 1: the O projection reads its input (attention output) from L2, not smem
  uint64_t *trace;             // optional: CTA 0 globaltimer at each grid barrier (exit, entry)
  uint32_t *trace_cta;         // optional: [kTraceMax][grid][kTraceCtaWords] low 32 bits of globaltimer
                               // per CTA (see cruise_epoch_read_trace_cta)
  uint64_t timeout_ns;         // bound of every spin wait
  uint32_t l2_ahead;           // bytes of weights prefetched into L2 beyond the ring (0: off)
  uint32_t l2_hints;           // bit 0: weight copies into the ring mark their L2 lines evict-first;
                               // bit 1: the run-ahead prefetch marks its lines evict-last
  // tensor parallelism (tp_size 1: off).  Every rank's exchange block is
  // mapped into every other rank (peer memory over NVLink); tp_peer[r] is rank r's.
  int32_t tp_size, tp_rank;
  TpExchange *const *tp_peer;  // device array [tp_size] of the ranks' exchange blocks
  TpExchange *tp_local;
  uint32_t tp_seq_base;        // launch-unique base of the exchange sequence numbers
  uint32_t launch_id;          // epochs launched by this engine, this one included
  StreamRing *stream;          // device view of the host-mapped egress ring (nullptr: off)
  int32_t mode;                // kModeEpoch, or kModeDecoderStep: one decoder call, no controller
};

}  // namespace cruise
