/*
 * cruise_epoch.h -- C ABI of the B200 resident decode-epoch engine.
 *
 * Plain C types only: every buffer is caller-owned host memory unless a
 * comment says otherwise, sizes are in bytes, and no entry point takes or
 * returns a framework type.  One engine owns one CUDA device, the model
 * weights, the resident paged K/V cache and the per-row resident state.
 *
 * Two layers of entry points:
 *   1. resident_epoch_create / _execute / _destroy keep the exact signatures
 *      of the reference host bridge (native/resident_epoch_bridge.h:24-45) so
 *      an existing ctypes / C caller binds them unchanged.
 *   2. cruise_epoch_* expose the engine directly: an explicit model geometry,
 *      weight loading, and the 8-input / 2-output epoch ABI of the reference's
 *      device controller (controller/g4c_b4_resident_epoch.cpp:40-49,296-324)
 *      with an explicit block table.
 */
#ifndef CRUISE_EPOCH_H
#define CRUISE_EPOCH_H

#include <stdint.h>

#include "cruise_protocol.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ---- reference-compatible bridge (native/resident_epoch_bridge.h) ------- */

#pragma pack(push, 1)
/* Device-IPC import metadata, byte-identical to the reference struct
 * (native/resident_epoch_bridge.h:8-21).  On CUDA each 64-byte key holds a
 * cudaIpcMemHandle_t of the exporting process's K or V cache allocation. */
typedef struct ResidentEpochIpcMetadata {
  uint64_t magic;
  uint32_t version;
  uint32_t import_mask;
  uint64_t source_bytes;
  int32_t row_generations[4];
  int32_t block_ids[4];
  uint64_t source_offsets[56];
  char keys[56][64];
} ResidentEpochIpcMetadata;
#pragma pack(pop)

/* Replaces resident_epoch_create (native/resident_epoch_bridge.cpp:360-422).
 *   air_path            model preset: "qwen2.5-7b" or "tiny"
 *   graph_config        ignored (may be NULL); kept for signature parity
 *   func_config         ignored (may be NULL)
 *   external_weight_dir "synthetic:<seed>" for seeded random-init weights, or a
 *                       directory holding one raw bf16 file "<tensor name>.bin"
 *                       per checkpoint tensor (HF names, row-major)
 *   tiling_path         optional 72-byte tiling blob (accepted, unused)
 * status: 0 ok, 1 bad arguments / engine already active, 2 tiling file,
 *         3 CUDA init, 4 weight load, 5 model geometry, 6 device memory. */
void *resident_epoch_create(const char *air_path, const char *graph_config,
                            const char *func_config,
                            const char *external_weight_dir,
                            const char *tiling_path, int32_t *status);

/* Replaces resident_epoch_execute (native/resident_epoch_bridge.cpp:424-649).
 * Same arguments, same transport statuses (10 bad args, 11 bad row, 12 active
 * count, 13 transfer file, 30 submit, 31 completion, 33 executed range,
 * 34 import checksum, 35 device IPC import) and the same commit-state moves
 * (0 -> 1 before submission -> 2 after a valid completion).  Row r owns the
 * blocks r*blocks_per_row + j, as in the reference bridge (:524-532).
 * output_token_ids is [4][8] row-major ([row][step]).  One addition: a
 * nonzero transfer_id with neither a transfer path nor IPC metadata imports
 * the rows of the last resident_epoch_prefill (13 when none is pending). */
int32_t resident_epoch_execute(
    void *opaque, int32_t request_count, int32_t max_steps,
    const int64_t *input_token_ids, const int64_t *input_positions,
    const int32_t *input_sequence_lengths, const int32_t *input_eos_token_ids,
    const int32_t *input_row_generations, int64_t *output_token_ids,
    int32_t *output_executed, int32_t *output_row_generations,
    int32_t *output_model_calls, int32_t *output_device_status,
    int32_t *output_feed_calls, int32_t *output_fetch_calls,
    int32_t *output_commit_state, int32_t *output_kv_import_checksum,
    int64_t *output_wall_us, int64_t *output_native_cpu_us,
    int64_t *output_declared_input_bytes,
    int64_t *output_declared_output_bytes, const char *transfer_path,
    uint64_t transfer_id, const ResidentEpochIpcMetadata *ipc_metadata);

/* Replaces resident_epoch_destroy (native/resident_epoch_bridge.cpp:651-670). */
void resident_epoch_destroy(void *opaque);

/* No reference counterpart: the device route for what the reference does as
 * a host prefill plus a one-shot KV import.  Runs cruise_epoch_prefill on the
 * bridge's engine for the prompts in prompt_tokens [4][stride] (row-major),
 * prompt_lens[r] in [0, min(stride, block_size)].  Rows with at least 2
 * tokens are then pending: the next resident_epoch_execute on this handle
 * called with transfer_path NULL, ipc_metadata NULL and a nonzero transfer_id
 * imports them from the device (Adler-32 proof in output_kv_import_checksum)
 * and decodes each from position len-1 with token prompt[len-1].  Every
 * pending row must run in that epoch (nonzero generation), else it returns 13
 * (and 11 if its position is not len-1); without a pending prefill it
 * returns 13 too.  Another import (a transfer
 * file or device IPC) discards the pending rows.  Returns 0, 10 bad
 * arguments (no row with 2 or more tokens), 11 a prompt longer than the
 * block size or a token outside the vocabulary, 30 a device failure. */
int32_t resident_epoch_prefill(void *opaque, const int64_t *prompt_tokens,
                               const int32_t *prompt_lens, int32_t stride);

/* ---- engine API ---------------------------------------------------------- */

/* Qwen2 geometry plus the paged-KV layout.  The static batch is 4 rows and an
 * epoch runs at most 8 steps, as in the reference (controller :16-17).
 * Replaces the hard-coded constants of controller/g4c_b4_resident_epoch.cpp:13-38. */
typedef struct CruiseModelConfig {
  int32_t num_layers;
  int32_t hidden;
  int32_t num_heads;
  int32_t num_kv_heads;
  int32_t head_dim;
  int32_t intermediate;
  int32_t vocab;
  float rms_eps;
  float rope_theta;
  int32_t block_size;      /* tokens per KV block */
  int32_t blocks_per_row;  /* logical capacity = block_size * blocks_per_row */
  int32_t num_blocks;      /* physical blocks in the resident cache */
  int32_t configured_eos;  /* EOS written for empty rows by the bridge */
  int32_t reserved[7];
} CruiseModelConfig;

/* Fills *cfg with a preset ("qwen2.5-7b" or "tiny"); returns 0 or -1. */
int32_t cruise_epoch_preset(const char *name, CruiseModelConfig *cfg);

/* Creates an engine on `device` with all device memory allocated and zeroed.
 * status as for resident_epoch_create.  Any number of engines may coexist
 * (one per device for data-parallel cohorts). */
void *cruise_epoch_create(const CruiseModelConfig *cfg, int32_t device,
                          int32_t *status);
void cruise_epoch_destroy(void *engine);

/* Tensor parallelism (no counterpart in the reference: its 2/4/8-device
 * sharding of the same epoch).  One process per GPU creates rank `tp_rank` of
 * `tp_size` (1, 2, 4 or 8): query heads, KV heads (shared by tp_size / KV-heads ranks
 * when tp_size exceeds them), intermediate rows and vocabulary rows are split
 * over the ranks; the residual stream, the embedding and the epoch control
 * are replicated.  The O and down projections are all-reduced inside the epoch
 * kernel through peer memory, the argmax across vocabulary shards likewise.
 * Tensors passed to cruise_epoch_set_weight / _get_weight and the KV cache of
 * _read_kv / _write_kv are this rank's shards, the logits of cruise_epoch_run
 * hold this rank's vocabulary rows at their global positions; the import
 * payload stays whole and history / control output are the same on every rank.
 * Before the first epoch every rank exports its exchange block with
 * cruise_epoch_tp_handle (a 64-byte cudaIpcMemHandle_t), the handles are
 * gathered in rank order (any host channel) and passed to
 * cruise_epoch_tp_connect.  All ranks must then run the same epochs; a rank
 * that does not makes the others' epoch end with status 207 (device waits are
 * bounded at 20 s under tensor parallelism). */
void *cruise_epoch_create_tp(const CruiseModelConfig *cfg, int32_t device,
                             int32_t tp_rank, int32_t tp_size,
                             int32_t *status);
int32_t cruise_epoch_tp_handle(void *engine, void *handle_out);
/* The shard of rank tp_rank of tp_size without creating an engine (host only):
 * shard_out[8] = {q0, nq, kv0, nkv, i0, ni, v0, nv} -- first query head and
 * count, first KV head and count, intermediate rows, vocabulary rows.
 * Returns 0, or -1 when the model does not split over tp_size ranks. */
int32_t cruise_epoch_tp_shard(const CruiseModelConfig *cfg, int32_t tp_rank,
                              int32_t tp_size, int32_t *shard_out);
int32_t cruise_epoch_tp_connect(void *engine, const void *handles);

/* Seeded random-init weights generated on the device: every tensor element is
 * bf16(0.02-scaled Irwin-Hall(4) sum of a splitmix64 hash of (seed, tensor,
 * index)).  Returns 0 or a CUDA error code. */
int32_t cruise_epoch_init_synthetic(void *engine, uint64_t seed, double stddev);

/* Copies one checkpoint tensor (HF name, row-major bf16) into the engine's
 * layout / out of it.  bytes must equal the tensor size.  0 on success,
 * -1 unknown name or size, else a CUDA error code. */
int32_t cruise_epoch_set_weight(void *engine, const char *name,
                                const void *host_bf16, uint64_t bytes);
int32_t cruise_epoch_get_weight(void *engine, const char *name, void *host_bf16,
                                uint64_t bytes);

/* Overrides the RoPE tables: bf16 cos and sin, [capacity][head_dim]. */
int32_t cruise_epoch_set_rope_table(void *engine, const uint16_t *cos_bf16,
                                    const uint16_t *sin_bf16, uint64_t bytes);

/* Whole resident K (or V) cache, bf16 [layers][num_blocks][block_size]
 * [kv_heads][head_dim]: copy out / in.  0 or a CUDA error code. */
int32_t cruise_epoch_read_kv(void *engine, void *key_host, void *value_host,
                             uint64_t bytes_each);
int32_t cruise_epoch_write_kv(void *engine, const void *key_host,
                              const void *value_host, uint64_t bytes_each);

/* One resident epoch through the 8-input / 2-output ABI of the reference's
 * device controller, entirely on the GPU (one submission, no per-token host
 * round trip).  Inputs (host): token i64[4], position i64[4], seq_len i32[4],
 * slot i32[4], active i32[4], block_table i32[4*blocks_per_row], tiling
 * u8[72] (may be NULL), control i32[11] = [K, eos x4, sampling, variant
 * (|0x100|mask to import), generation x4].  import_payload: when importing,
 * [K|V][layers][4 rows][block_size][kv_heads][head_dim] bf16 on the host, or
 * NULL with import_bytes 0 to import what cruise_epoch_prefill computed.
 * forced_tokens: NULL for greedy decoding, or i64[8][4] step-major where an
 * entry >= 0 replaces the argmax of that row at that step (teacher forcing:
 * the device prefill of a prompt runs as forced epochs).
 * Outputs (host): history i64[8][4] step-major (-1 filled) and control_out
 * i32[28] (layout of controller :296-324).  logits_out, if not NULL, receives
 * f32 [8][4][vocab] (steps never run stay untouched).  Returns 0 when the
 * epoch ran (the device status is control_out[3]) or a CUDA error code. */
int32_t cruise_epoch_run(void *engine, const int64_t *token,
                         const int64_t *position, const int32_t *seq_len,
                         const int32_t *slot, const int32_t *active,
                         const int32_t *block_table, const uint8_t *tiling,
                         const int32_t *control, const void *import_payload,
                         uint64_t import_bytes, const int64_t *forced_tokens,
                         int64_t *history, int32_t *control_out,
                         float *logits_out);

/* No counterpart in the reference.  The same greedy epoch as cruise_epoch_run
 * for callers that must not allocate device memory once they are serving:
 * a host whose device memory is all handed to its own pool up front (a
 * serving worker that reserves most of HBM for its KV pool at start-up, where
 * a cudaMalloc behind its back fails or fragments the pool), or a runtime
 * whose policy forbids allocation after warm-up.  This call allocates
 * nothing: the epoch's scratch (inputs/outputs block, grid-barrier counters,
 * activations, split-tile partials, argmax partials) lives in one static
 * 1 MiB device array compiled into this library, which every GPU that loads
 * the library holds until the process exits.  The engine's weights, KV cache
 * and resident row state are used as by cruise_epoch_run, so both calls may
 * be mixed on one engine.
 * Arguments mean what they mean for cruise_epoch_run (host arrays; no tiling,
 * forced tokens or logits).  KV imports are not accepted here.
 * The first call on a device looks up the array's device address (once per
 * device) and keeps it for the life of the process, so the call must not be
 * used after a cudaDeviceReset of that device; make that first call before
 * any stream capture.  The call returns after the epoch completed (it waits
 * for the engine's stream).  Every call, on every engine of the process,
 * shares the one array and clears it first: calls that overlap in time (two
 * threads, two engines on one GPU) race and must be serialised by the caller.
 * cruise_epoch_last_timing reports this call like cruise_epoch_run, and a
 * device status 207 names the wait that gave up in cruise_epoch_last_error.
 * Returns 0 when the epoch ran (device status in control_out[3]), -1 for a
 * NULL argument, -2 when the model's scratch exceeds the 1 MiB array, -3 for
 * an import request, -4 for a tensor-parallel engine, or a CUDA error code;
 * cruise_epoch_last_error explains -2, -3 and -4. */
int32_t cruise_epoch_run_noalloc(void *engine, const int64_t *token,
                                 const int64_t *position,
                                 const int32_t *seq_len, const int32_t *slot,
                                 const int32_t *active,
                                 const int32_t *block_table,
                                 const int32_t *control, int64_t *history,
                                 int32_t *control_out);

/* One decoder step through the 9-input / 4-output decoder ABI of the
 * reference's decode graph (config/graph_config.json:6-16; the call the
 * device controller makes once per step, controller/g4c_b4_resident_epoch.cpp
 * :485-498, and the host-loop runner K times per epoch,
 * g4c_b4_epoch_runner.cpp:245-382).  No controller runs: the caller decides
 * tokens, termination and slots between calls.
 * Inputs, in the ABI's order (host arrays): token i64[4] (the ABI's [4,1]),
 * position i64[4], seq_len i32[4] ([4,1]), key_cache, slot i32[4], active
 * i32[4], block_table i32[4*blocks_per_row], value_cache, tiling u8[72]
 * (may be NULL; accepted and unused).
 * key_cache / value_cache: device bf16 [layers][num_blocks][block_size]
 * [kv_heads][head_dim] on the engine's device, 16-byte aligned, updated in
 * place (the ABI's K and V outputs); both NULL for the engine's resident
 * caches.
 * Outputs (host): logits_out f32 [4][vocab], next_position_out i64[4] =
 * position + 1 for active rows, position otherwise.
 * For active rows the step computes exactly what the reference decoder does
 * (batched_decoder_step.py:277-417): the new K/V are written at slot[row]
 * and attention covers positions < seq_len.  Rows with active 0 write no K/V
 * and keep their position; their logits are not computed from attention and
 * must not be used (the reference's callers never read them, controller
 * :547-552).
 * Returns 0, -1 for invalid arguments (a token outside the vocabulary, an
 * active row whose position is outside the capacity or whose slot is not its
 * position's block-table slot, a block-table entry outside the cache, a
 * sequence length above the capacity, caches that are not device memory of
 * the engine's device), -3 when a device-side wait gave up, -4 for a
 * tensor-parallel engine, or a CUDA error code; cruise_epoch_last_error
 * explains -1, -3 and -4. */
int32_t cruise_decoder_step(void *engine, const int64_t *token,
                            const int64_t *position, const int32_t *seq_len,
                            void *key_cache, const int32_t *slot,
                            const int32_t *active, const int32_t *block_table,
                            void *value_cache, const uint8_t *tiling,
                            float *logits_out, int64_t *next_position_out);

/* Device time of the last epoch (or decoder step) in microseconds (CUDA
 * events around the epoch kernel) and the number of kernels it launched. */
int32_t cruise_epoch_last_timing(void *engine, double *device_us,
                                 int32_t *kernel_launches);

/* Phase trace (tracing / profiling aid): when enabled, each epoch records, per
 * grid barrier j (1-based, in launch order; at most 2048 per epoch), globaltimer
 * nanoseconds in six series:
 *   0  CTA 0 left barrier j (every CTA had arrived)
 *   1  CTA 0 arrived at barrier j (finished its share of the phase)
 *   2  CTA 0 had staged the phase's activations (projection phases)
 *   3  CTA 0's warp 0 consumed its last weight tile (projection phases)
 *   4  the last CTA arrived at barrier j
 *   5  not a time stamp: nanoseconds CTA 0's epilogue waited for the other
 *      ranks' partials in phase j (O and down of a tensor-parallel engine;
 *      0 otherwise)
 * cruise_epoch_read_trace copies `count` entries of one series.
 * enable = 2 also records, for EVERY CTA and barrier j, eight words, the low
 * 32 bits of globaltimer unless noted: [0] the CTA left barrier j, [1] it had
 * staged the activations of the phase ending at j (projection phases), [2] its
 * warp 0 consumed its last weight tile there, [3] it arrived at barrier j;
 * its epilogue warp [4] started the phase, [5] waited that many ns for the
 * stream-K partner's partial sums, [6] finished its last row group, [7] had
 * fenced its outputs, [8] received the consumers' last partial sums; [9] its
 * last consumer warp consumed its last weight tile; RMSNorm staging (QKV,
 * gate/up, lm_head): [10] the residual rows had arrived, [11] the sums of
 * squares were shared.
 * cruise_epoch_read_trace_cta copies `barriers` x ctas x 12 words (barrier-
 * major) and reports the CTA count; 0 = no record. */
int32_t cruise_epoch_set_trace(void *engine, int32_t enable);
int32_t cruise_epoch_read_trace(void *engine, int32_t series, uint64_t *ns,
                                int32_t count);
int32_t cruise_epoch_read_trace_cta(void *engine, uint32_t *stamps,
                                    int32_t barriers, int32_t *ctas);

/* Batched device prefill (the reference prefills on the host and imports the
 * KV; here the prompts run through the model on the GPU in one pass per
 * layer).  prompt_tokens is [4][stride] (row-major), prompt_lens[r] in
 * [0, block_size] (0: row not prefilled).  Computes the K and V of tokens
 * 0..len-2 of every row at positions 0..len-2 into the engine's import
 * staging buffer -- [K|V][layers][4][block_size][kv_heads][head_dim], the
 * import payload format -- and keeps it there: the next cruise_epoch_run with
 * the import flag and import_payload NULL / import_bytes 0 imports it (one-shot
 * device import with the Adler-32 proof) and decodes from position len-1 with
 * token prompt[len-1].  The projections run as the engine's own tcgen05
 * GEMMs, reading the resident tiled weights through TMA (no second copy of
 * the weights; the first call allocates the activation buffers, kept until
 * destroy); attention, norms, rope and SwiGLU follow the decoder step's
 * rounding points.  Geometry limits: block_size <= 128, head size 64 or
 * 128, at most 8 query heads per KV head, intermediate and hidden sizes
 * divisible by 8, hidden size at most 8192 (others return -1 with the reason
 * in cruise_epoch_last_error).  0, -1 bad arguments, -2 library failure, -4
 * tensor-parallel engine, or a CUDA error code; after a failure in the first
 * call's set-up the next call starts the set-up over. */
int32_t cruise_epoch_prefill(void *engine, const int64_t *prompt_tokens,
                             const int32_t *prompt_lens, int32_t stride);

/* Streaming token egress (a reference evaluation item: stream without K=1).
 * With streaming enabled, every decode step of an epoch publishes that step's
 * four tokens (-1 for rows that did not run) to host-mapped pinned memory as
 * soon as the device decided them, while cruise_epoch_run still waits for the
 * epoch.  cruise_epoch_stream_next_id gives the id the next epoch of this
 * engine will carry; another host thread then calls cruise_epoch_stream_poll
 * with it: returns how many steps of that epoch were published so far (0
 * before the first) and copies their tokens, step-major, into tokens_out
 * [8][4]; -1 if streaming was never enabled.  Poll takes no lock. */
int32_t cruise_epoch_stream_enable(void *engine, int32_t enable);
uint32_t cruise_epoch_stream_next_id(void *engine);
int32_t cruise_epoch_stream_poll(void *engine, uint32_t launch_id,
                                 int64_t *tokens_out);

/* Last CUDA error string of this engine (static storage).  With engine NULL:
 * why the calling thread's last cruise_epoch_create / _create_tp returned
 * NULL (the failing step and CUDA error), "" after a successful create. */
const char *cruise_epoch_last_error(void *engine);

#ifdef __cplusplus
}
#endif

#endif /* CRUISE_EPOCH_H */
