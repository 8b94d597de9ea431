// engine.cu -- host side of the B200 resident decode-epoch engine and its C ABI
// (include/cruise_epoch.h): device memory, seeded weight synthesis, weight
// loading, the one-launch epoch, and the reference-compatible bridge
// resident_epoch_create / _execute / _destroy.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <array>
#include <atomic>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <map>
#include <mutex>
#include <string>
#include <time.h>
#include <vector>

#include "../../include/cruise_epoch.h"
#include "epoch_kernel.cuh"
#include "prefill.cuh"
#include "prefill_gemm.cuh"

namespace cruise {
namespace {

constexpr long kDefaultL2AheadKb = 128;   // L2 run-ahead of the weight stream per CTA
constexpr uint32_t kDefaultL2Hints = 1;   // weight copies into the ring mark their L2 lines evict-first

constexpr int kLayerTensors = 12;  // per-layer checkpoint tensors, in id order
const char *const kLayerKeys[kLayerTensors] = {
    "input_layernorm.weight", "post_attention_layernorm.weight",
    "self_attn.q_proj.weight", "self_attn.q_proj.bias",
    "self_attn.k_proj.weight", "self_attn.k_proj.bias",
    "self_attn.v_proj.weight", "self_attn.v_proj.bias",
    "self_attn.o_proj.weight", "mlp.gate_proj.weight",
    "mlp.up_proj.weight",      "mlp.down_proj.weight"};

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// ---- seeded weight synthesis (splitmix64 -> Irwin-Hall(4) -> bf16) -------------
constexpr uint64_t kGamma = 0x9E3779B97F4A7C15ull;
constexpr uint64_t kKeyMul = 0xD1B54A32D192ED03ull;

__host__ __device__ inline uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

enum SynthMode : int32_t { kPlain = 0, kQkvRows = 1, kGateUp = 2, kDownPad = 3, kRowsPad = 4 };

struct SynthMap {
  int32_t mode;
  int32_t ids[3];       // tensor ids (q,k,v for kQkvRows; gate,up for kGateUp)
  int64_t cols;         // row length of the canonical tensor(s)
  int64_t rows0, rows1; // q rows / k rows (kQkvRows); valid rows (kRowsPad)
  int64_t dst_cols;     // packed row length (kDownPad: columns [off0, off0 + rows0) of each row, zeros up to it)
  int64_t off0, off1;   // shard offsets into the canonical tensor (tensor parallelism):
                        // q row / k,v row (kQkvRows), intermediate row (kGateUp),
                        // column (kDownPad), vocabulary row (kRowsPad)
  int32_t tiled;        // destination is a tiled matrix with dst_cols columns
  int32_t kc;           // its tile width
};

__device__ __forceinline__ uint16_t synth_value(uint64_t key, int64_t index, float scale) {
  const uint64_t h = mix64(key + static_cast<uint64_t>(index + 1) * kGamma);
  const int32_t sum = static_cast<int32_t>((h & 0xFFFF) + ((h >> 16) & 0xFFFF) + ((h >> 32) & 0xFFFF) +
                                           (h >> 48));
  const float centred = static_cast<float>(2 * sum - 262140);
  const float v = __fmul_rn(centred, scale);
  return __bfloat16_as_ushort(__float2bfloat16_rn(v));
}

__global__ void synth_kernel(uint16_t *dst, int64_t count, SynthMap map, uint64_t seed, float scale) {
  for (int64_t d = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; d < count;
       d += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    int64_t e = d;   // logical row-major index of the packed matrix
    if (map.tiled) {
      const int64_t kc = map.kc;
      const int64_t tile = d / (kRows * kc), rem = d % (kRows * kc);
      const int64_t r = rem / kc, pu = (rem % kc) >> 3, el = rem & 7;
      const int64_t KT = map.dst_cols / kc;
      const int64_t n = (tile / KT) * kRows + r;
      const int64_t k = (tile % KT) * kc + ((pu ^ (r & 7)) << 3) + el;
      e = n * map.dst_cols + k;
    }
    int32_t id = map.ids[0];
    int64_t idx = e;
    bool zero = false;
    switch (map.mode) {
      case kQkvRows: {
        const int64_t r = e / map.cols, c = e % map.cols;
        if (r < map.rows0) { id = map.ids[0]; idx = (map.off0 + r) * map.cols + c; }
        else if (r < map.rows0 + map.rows1) { id = map.ids[1]; idx = (map.off1 + r - map.rows0) * map.cols + c; }
        else { id = map.ids[2]; idx = (map.off1 + r - map.rows0 - map.rows1) * map.cols + c; }
        break;
      }
      case kGateUp: {
        const int64_t R = e / map.cols, c = e % map.cols;
        const int64_t blk = R / 16, rr = R % 16;
        id = rr < 8 ? map.ids[0] : map.ids[1];
        idx = (map.off0 + blk * 8 + (rr & 7)) * map.cols + c;
        break;
      }
      case kDownPad: {
        const int64_t r = e / map.dst_cols, c = e % map.dst_cols;
        zero = c >= map.rows0;
        idx = r * map.cols + map.off0 + c;
        break;
      }
      case kRowsPad: {
        const int64_t r = e / map.cols, c = e % map.cols;
        zero = r >= map.rows0;
        idx = (map.off0 + r) * map.cols + c;
        break;
      }
      default:
        break;
    }
    const uint64_t key = mix64(seed * kGamma + static_cast<uint64_t>(id + 1) * kKeyMul);
    dst[d] = zero ? 0 : synth_value(key, idx, scale);
  }
}

// Canonical row i of a checkpoint tensor -> logical row of the packed matrix.
enum RowMap : int32_t { kRowOffset = 0, kRowGate = 1, kRowUp = 2 };

__device__ __forceinline__ int64_t packed_row(int32_t map, int64_t i, int64_t offset) {
  if (map == kRowGate) return (i / 8) * 16 + (i % 8);
  if (map == kRowUp) return (i / 8) * 16 + 8 + (i % 8);
  return offset + i;
}

// Moves one canonical [rows][cols] tensor into (to_tiled) or out of a tiled
// matrix with K columns and tile width kc.
__global__ void tile_copy_kernel(uint16_t *tiled, uint16_t *canonical, int64_t rows, int64_t cols, int32_t map,
                                 int64_t offset, int64_t K, int32_t kc, int32_t to_tiled) {
  const int64_t count = rows * cols;
  for (int64_t e = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; e < count;
       e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t i = e / cols, c = e % cols;
    const int64_t dst = tiled_offset(packed_row(map, i, offset), c, K, kc);
    if (to_tiled) {
      tiled[dst] = canonical[e];
    } else {
      canonical[e] = tiled[dst];
    }
  }
}

struct Region {
  uint16_t *ptr = nullptr;   // packed device buffer
  int64_t elems = 0;
};

// Activation buffers of the batched prefill, built on the first
// cruise_epoch_prefill (the decode epoch never needs them).  The projections
// read the engine's own tiled weights.
struct PrefillState {
  void *work = nullptr;
  int max_tokens = 0;
  bf16 *h = nullptr, *x = nullptr, *q = nullptr, *attn = nullptr, *act = nullptr;
  bf16 *y = nullptr;           // a projection's bf16 output [T][H] (O without k splits)
  float *acc = nullptr;        // fp32 k-range partial sums [split][T][N]
  int64_t *tok = nullptr;
  int32_t *row = nullptr, *pos = nullptr;
  uint32_t *error = nullptr;   // site of a tensor-core GEMM wait that ran out (0: none)
  bool chain = true;           // kernels launched as programmatic dependents (CRUISE_PREFILL_PDL=0: plain)
  int narrow_tile = 0;         // token tile cap of QKV, O and down (CRUISE_PREFILL_TTILE; 0: all tokens)
  int force_split = 0;         // their split count (CRUISE_PREFILL_SPLIT; 0: the cost model's)
  bool w_evict_first = true;   // GEMM weight copies evict-first in L2 (CRUISE_PREFILL_WHINT=0: no hint)
  int stage_cap = 0;           // ring depth cap of the GEMM (CRUISE_PREFILL_STAGES; 0: as many as fit)
  bool p_evict_last = true;    // partial sums stored evict-last in L2 (CRUISE_PREFILL_PHINT=0: no hint)
  bool gemm_attr = false;      // the GEMM's shared-memory limit has been raised
  int gemm_pairs = 0;          // resident CTA pairs of the GEMM (0: not yet asked)
  // profiling (CRUISE_PREFILL_TRACE=1): %globaltimer marks of the first
  // kTraceLaunches GEMM launches of a prefill, summarised on stderr
  uint64_t *trace = nullptr;
  int trace_calls = 0;
  int trace_grid[8] = {};
};
constexpr int kTraceLaunches = 8;

struct Engine {
  CruiseModelConfig cfg{};
  ModelDims m{};
  int device = 0;
  cudaStream_t stream = nullptr;
  cudaEvent_t ev0 = nullptr, ev1 = nullptr;
  int sms = 0;
  int stages = 0;
  int xs_stride = 0;
  uint32_t l2_ahead = 0;   // bytes of L2 run-ahead per CTA (CRUISE_L2_AHEAD_KB)
  uint32_t l2_hints = 0;   // L2 eviction-priority hints of the weight stream (CRUISE_L2_HINTS)
  int down_xglobal = 0;
  int o_xglobal = 0;
  uint64_t *trace = nullptr;     // per-launch phase timestamps (optional)
  bool trace_on = false;
  uint32_t *trace_cta = nullptr; // per-CTA phase timestamps (allocated when first enabled)
  bool trace_cta_on = false;
  size_t smem = 0;
  // device memory
  void *weights = nullptr;   // one allocation for every weight tensor
  size_t weight_bytes = 0;
  std::vector<LayerWeights> layers;
  LayerWeights *d_layers = nullptr;
  bf16 *embed = nullptr, *final_norm = nullptr, *lm_head = nullptr;
  void *state = nullptr;     // caches, activations, control blocks
  bf16 *key_cache = nullptr, *value_cache = nullptr;
  bf16 *rope_cos = nullptr, *rope_sin = nullptr;
  bf16 *h = nullptr, *qkv = nullptr, *attn = nullptr, *act = nullptr;
  uint64_t *partials = nullptr;   // tagged split row-group partials, right after d_sync
  float *arg_val = nullptr, *logits = nullptr;
  int32_t *arg_idx = nullptr, *arg_bad = nullptr;
  EpochIO *d_io = nullptr;
  ResidentState *d_res = nullptr;
  EpochWork *d_work = nullptr;
  SyncState *d_sync = nullptr;
  uint8_t *d_payload = nullptr;   // import staging, allocated on first import
  size_t payload_bytes = 0;
  EpochIO *h_io = nullptr;        // pinned staging
  float last_ms = 0.f;
  int32_t last_launches = 0;
  std::string last_error;
  std::mutex execute_mutex;
  std::array<uint8_t, kTilingBytes> tiling{};
  // tensor parallelism
  int tp_rank = 0, tp_size = 1;
  TpExchange *xchg = nullptr;              // this rank's exchange block (IPC-exported)
  TpExchange **d_peers = nullptr;          // device array of every rank's block
  std::vector<void *> opened;              // peer blocks opened through IPC
  bool tp_connected = false;
  std::atomic<uint32_t> launches{0};       // epochs launched (exchange sequence base, egress launch id)
  StreamRing *h_stream = nullptr;          // host-mapped egress ring (allocated on first enable)
  StreamRing *d_stream = nullptr;          // its device view
  bool stream_on = false;
  PrefillState *prefill = nullptr;
  bool payload_ready = false;   // d_payload holds a prefilled cohort for the next import epoch
  uint64_t tp_timeout_ns = 20000000000ull;   // device waits on other ranks (CRUISE_TP_TIMEOUT_MS)
};

// Every host<->device copy runs on the engine's own (non-blocking) stream and is
// waited for: a pageable-memory cudaMemcpy on the legacy stream may return before
// its DMA lands, and the engine's stream does not order after the legacy stream.
cudaError_t copy_sync(Engine *e, void *dst, const void *src, size_t bytes, cudaMemcpyKind kind) {
  cudaError_t err = cudaMemcpyAsync(dst, src, bytes, kind, e->stream);
  if (err == cudaSuccess) err = cudaStreamSynchronize(e->stream);
  return err;
}

int32_t set_err(Engine *e, cudaError_t err, const char *what) {
  if (err != cudaSuccess && e != nullptr) {
    e->last_error = std::string(what) + ": " + cudaGetErrorString(err);
  }
  return static_cast<int32_t>(err);
}

bool valid_config(const CruiseModelConfig &c) {
  if (c.num_layers < 1 || c.num_layers > 64 || c.hidden < 64 || c.hidden % 64 != 0) return false;
  if (c.hidden > 4096) return false;   // RMSNorm staging: 2 x 8 elements per thread and row
  if (c.num_heads < 1 || c.num_kv_heads < 1 || c.num_heads % c.num_kv_heads != 0) return false;
  if (c.num_kv_heads > kMaxKvGroups) return false;   // one QKV completion counter per KV head
  if (c.head_dim != 64 && c.head_dim != 128) return false;
  if (c.num_heads * c.head_dim != c.hidden) return false;
  if (c.intermediate < 8 || c.intermediate % 8 != 0) return false;
  if (c.vocab < 2) return false;
  if (c.block_size < 1 || c.blocks_per_row < 1 || c.blocks_per_row > kMaxBlocksPerRow) return false;
  if (c.num_blocks < kBatch * c.blocks_per_row || c.num_blocks > 256) return false;
  if (((2 * c.num_kv_heads * c.head_dim) % kRows) != 0) return false;
  // Adler-32 splits a block over 256 threads in 16-byte pieces
  if ((static_cast<int64_t>(c.block_size) * c.num_kv_heads * c.head_dim * 2) % (256 * 16) != 0) return false;
  if (c.configured_eos < 0 || c.configured_eos >= c.vocab) return false;
  return true;
}

// Shard of tensor-parallel rank `rank` of `size`: query heads [q0, q0+nq) and
// KV heads [kv0, kv0+nkv) (a rank holds whole KV groups when size <= KV heads,
// else size / KV-heads ranks share one KV head and split its query heads,
// the first ranks of a group taking one more), intermediate rows [i0, i0+ni)
// and vocabulary rows [v0, v0+nv).
struct TpGeom {
  int q0, nq, kv0, nkv, i0, ni, v0, nv;
};

bool tp_geometry(const CruiseModelConfig &c, int rank, int size, TpGeom &g) {
  // 1, 2, 4 or 8 ranks (the kernel's cross-rank reduction is unrolled for those)
  if ((size != 1 && size != 2 && size != 4 && size != 8) || rank < 0 || rank >= size) return false;
  const int nq = c.num_heads, nkv = c.num_kv_heads, grp = nq / nkv;
  if (size <= nkv) {
    if (nkv % size != 0) return false;
    g.nkv = nkv / size;
    g.kv0 = rank * g.nkv;
    g.q0 = g.kv0 * grp;
    g.nq = g.nkv * grp;
  } else {
    if (size % nkv != 0) return false;
    const int per = size / nkv;   // ranks sharing one KV head
    if (grp < per) return false;
    const int part = rank % per, base = grp / per, extra = grp % per;
    g.kv0 = rank / per;
    g.nkv = 1;
    g.q0 = g.kv0 * grp + part * base + std::min(part, extra);
    g.nq = base + (part < extra ? 1 : 0);
  }
  if (c.intermediate % size != 0 || (c.intermediate / size) % 8 != 0) return false;
  g.ni = c.intermediate / size;
  g.i0 = rank * g.ni;
  const int vs = (c.vocab + size - 1) / size;
  g.v0 = rank * vs;
  g.nv = std::min(vs, c.vocab - g.v0);
  return g.nv > 0;
}

void fill_dims(Engine *e) {
  const CruiseModelConfig &c = e->cfg;
  ModelDims &m = e->m;
  TpGeom g{};
  tp_geometry(c, e->tp_rank, e->tp_size, g);   // validated by the caller
  m.L = c.num_layers;
  m.H = c.hidden;
  m.nq = g.nq;
  m.nkv = g.nkv;
  m.d = c.head_dim;
  m.q0 = g.q0;
  m.kv0 = g.kv0;
  m.nkv_all = c.num_kv_heads;
  m.Hq = g.nq * c.head_dim;
  // The O projection's input columns (this rank's query heads) are zero-padded
  // to a multiple of 512 where that adds at most a third and stays within H:
  // its tiles are then 512 wide, so all consumer warps multiply and the
  // attention output is read straight from L2, and at TP = 8 the two ranks
  // sharing a KV head (4 and 3 query heads) stream O shards of one shape.
  // One GPU (Hq = H = 3584) is unchanged.
  {
    const int32_t kq512 = static_cast<int32_t>(align_up(m.Hq, 512));
    m.Kq = kq512 <= c.hidden && static_cast<int64_t>(kq512) * 3 <= static_cast<int64_t>(m.Hq) * 4 ? kq512 : m.Hq;
  }
  m.I = g.ni;
  // intermediate columns zero-padded to a multiple of 512 (the down projection's
  // 512-wide tiles and its activation read straight from L2) when that adds at
  // most a tenth to the down weights, else to a multiple of 64
  const int64_t pad512 = static_cast<int64_t>(align_up(g.ni, 512));
  m.I_pad = static_cast<int32_t>(pad512 * 10 <= static_cast<int64_t>(g.ni) * 11 ? pad512 : align_up(g.ni, 64));
  m.V = c.vocab;
  m.v0 = g.v0;
  m.Vl = g.nv;
  m.V_pad = static_cast<int32_t>(align_up(g.nv, kRows));
  m.Nqkv = (g.nq + 2 * g.nkv) * c.head_dim;
  m.eps = c.rms_eps;
  m.sqrt_d = static_cast<float>(std::sqrt(static_cast<double>(c.head_dim)));
  m.bs = c.block_size;
  m.bpr = c.blocks_per_row;
  m.NB = c.num_blocks;
  m.C = c.block_size * c.blocks_per_row;
}

// Default RoPE tables: inv_freq = 1 / theta^(2i/d) and cos/sin of pos*inv_freq
// in fp32, rounded to bf16, following batched_decoder_step.py:212-216,235-240.
void default_rope(const Engine *e, std::vector<uint16_t> &cos_t, std::vector<uint16_t> &sin_t) {
  const int d = e->m.d, C = e->m.C;
  cos_t.resize(static_cast<size_t>(C) * d);
  sin_t.resize(static_cast<size_t>(C) * d);
  auto to_bf16 = [](float v) {
    uint32_t bits;
    std::memcpy(&bits, &v, 4);
    bits += 0x7FFFu + ((bits >> 16) & 1u);
    return static_cast<uint16_t>(bits >> 16);
  };
  for (int pos = 0; pos < C; ++pos) {
    for (int i = 0; i < d / 2; ++i) {
      const float expo = static_cast<float>(2 * i) / static_cast<float>(d);
      const float inv = 1.0f / std::pow(e->cfg.rope_theta, expo);
      const float f = static_cast<float>(pos) * inv;
      const uint16_t cv = to_bf16(static_cast<float>(std::cos(static_cast<double>(f))));
      const uint16_t sv = to_bf16(static_cast<float>(std::sin(static_cast<double>(f))));
      cos_t[static_cast<size_t>(pos) * d + i] = cos_t[static_cast<size_t>(pos) * d + i + d / 2] = cv;
      sin_t[static_cast<size_t>(pos) * d + i] = sin_t[static_cast<size_t>(pos) * d + i + d / 2] = sv;
    }
  }
}

void prefill_release(Engine *e);

void destroy_engine(Engine *e) {
  if (e == nullptr) return;
  cudaSetDevice(e->device);
  if (e->stream) cudaStreamSynchronize(e->stream);
  cudaFree(e->weights);
  cudaFree(e->state);
  cudaFree(e->d_layers);
  cudaFree(e->d_payload);
  for (void *ptr : e->opened) cudaIpcCloseMemHandle(ptr);
  cudaFree(e->d_peers);
  cudaFree(e->trace_cta);
  cudaFree(e->xchg);
  if (e->h_io) cudaFreeHost(e->h_io);
  if (e->h_stream) cudaFreeHost(e->h_stream);
  prefill_release(e);
  if (e->ev0) cudaEventDestroy(e->ev0);
  if (e->ev1) cudaEventDestroy(e->ev1);
  if (e->stream) cudaStreamDestroy(e->stream);
  delete e;
}

// why the calling thread's last create_engine returned null ("" after a success)
thread_local std::string g_create_error;

Engine *create_engine(const CruiseModelConfig &cfg, int device, int32_t *status, int tp_rank = 0,
                      int tp_size = 1) {
  g_create_error.clear();
  *status = 5;
  if (!valid_config(cfg)) {
    g_create_error = "unsupported model configuration";
    return nullptr;
  }
  TpGeom geom{};
  if (!tp_geometry(cfg, tp_rank, tp_size, geom)) {
    g_create_error = "no tensor-parallel sharding of this model over " + std::to_string(tp_size) + " ranks";
    return nullptr;
  }
  Engine *e = new Engine();
  e->cfg = cfg;
  e->device = device;
  e->tp_rank = tp_rank;
  e->tp_size = tp_size;
  fill_dims(e);
  const ModelDims &m = e->m;
  *status = 3;
  // records why creation stopped (read back through cruise_epoch_last_error(NULL))
  auto fail = [&](const char *what, bool destroy = true) -> Engine * {
    const cudaError_t err = cudaGetLastError();
    g_create_error = std::string(what) + (err != cudaSuccess ? std::string(": ") + cudaGetErrorString(err) : "");
    if (destroy) {
      destroy_engine(e);
    } else {
      delete e;
    }
    return nullptr;
  };
  if (cudaSetDevice(device) != cudaSuccess) return fail("cudaSetDevice", false);
  cudaDeviceProp prop{};
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return fail("cudaGetDeviceProperties", false);
  if (prop.major < 10) return fail("the engine is built for sm_100a (compute capability 10.x)", false);
  int coop = 0;
  cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, device);
  if (!coop) return fail("the device does not support cooperative launches", false);
  e->sms = std::min(prop.multiProcessorCount, kMaxCtas);
  if (cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking) != cudaSuccess ||
      cudaEventCreate(&e->ev0) != cudaSuccess || cudaEventCreate(&e->ev1) != cudaSuccess) {
    return fail("stream or event creation");
  }
  // shared memory geometry: the activation rows in smem hold the widest input of
  // the projections that stage it there; the down projection reads its input
  // from L2 instead when it runs one 64-wide k-step per consumer warp.
  e->down_xglobal = pick_kc(m.I_pad) == 64 * kConsumerWarps;
  {
    // the O projection reads the attention output straight from L2 when it
    // runs one 64-wide k-step per consumer warp (CRUISE_O_XGLOBAL=0 stages it)
    const char *env = std::getenv("CRUISE_O_XGLOBAL");
    e->o_xglobal = pick_kc(m.Kq) == 64 * kConsumerWarps && (env == nullptr || std::strtol(env, nullptr, 10) != 0);
  }
  const int kmax = e->down_xglobal ? m.H : std::max(m.H, m.I_pad);
  e->xs_stride = kmax + 8;
  if (const char *env = std::getenv("CRUISE_TP_TIMEOUT_MS")) {
    const long ms = std::strtol(env, nullptr, 10);
    if (ms > 0) e->tp_timeout_ns = static_cast<uint64_t>(std::min(ms, 600000L)) * 1000000ull;
  }
  {
    const char *env = std::getenv("CRUISE_L2_AHEAD_KB");
    const long kb = env != nullptr ? std::strtol(env, nullptr, 10) : kDefaultL2AheadKb;
    e->l2_ahead = static_cast<uint32_t>(std::min(std::max(kb, 0L), 4096L)) * 1024u;
    const char *hints = std::getenv("CRUISE_L2_HINTS");
    e->l2_hints = static_cast<uint32_t>(hints != nullptr ? std::strtol(hints, nullptr, 10) & 3 : kDefaultL2Hints);
  }
  // the attention unit's scratch aliases the activation rows and the reduction ring
  if (attn_scratch_bytes(m.d, m.C) >
      static_cast<size_t>(kBatch) * e->xs_stride * 2 + static_cast<size_t>(kRedSlots) * kConsumerWarps * 64 * 4) {
    return fail("the attention scratch does not fit the activation rows");
  }
  const size_t limit = prop.sharedMemPerBlockOptin;
  int stages = kMaxStages;
  while (stages > 2 && smem_bytes(stages, e->xs_stride) > limit) --stages;
  e->stages = stages;
  e->smem = smem_bytes(stages, e->xs_stride);
  if (e->smem > limit) {
    *status = 5;
    return fail("shared memory of the smallest stage ring exceeds the per-block limit");
  }
  if (cudaFuncSetAttribute(resident_epoch_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(e->smem)) != cudaSuccess) {
    return fail("cudaFuncSetAttribute(max dynamic shared memory)");
  }
  int per_sm = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, resident_epoch_kernel, kThreads, e->smem);
  if (per_sm < 1) return fail("the epoch kernel has no resident CTA per SM (registers or shared memory)");

  // ---- weights: one allocation ----
  *status = 6;
  const int64_t H = m.H, kv = static_cast<int64_t>(m.nkv) * m.d;
  std::vector<size_t> offs;
  size_t total = 0;
  auto take = [&](int64_t elems) {
    const size_t off = total;
    total = align_up(total + static_cast<size_t>(elems) * 2, 256);
    return off;
  };
  const size_t off_embed = take(static_cast<int64_t>(m.V) * H);
  struct LayerOff { size_t w_in, w_post, qkv_w, qkv_b, o_w, gu_w, down_w; };
  std::vector<LayerOff> lo(m.L);
  for (int l = 0; l < m.L; ++l) {
    lo[l].w_in = take(H);
    lo[l].w_post = take(H);
    lo[l].qkv_w = take(static_cast<int64_t>(m.Nqkv) * H);
    lo[l].qkv_b = take(m.Nqkv);
    lo[l].o_w = take(H * static_cast<int64_t>(m.Kq));
    lo[l].gu_w = take(2LL * m.I * H);
    lo[l].down_w = take(H * m.I_pad);
  }
  const size_t off_norm = take(H);
  const size_t off_lm = take(static_cast<int64_t>(m.V_pad) * H);
  (void)kv;
  e->weight_bytes = total;
  if (cudaMalloc(&e->weights, total) != cudaSuccess) return fail("weight allocation");
  cudaMemsetAsync(e->weights, 0, total, e->stream);
  uint8_t *wb = static_cast<uint8_t *>(e->weights);
  auto wp = [&](size_t off) { return reinterpret_cast<bf16 *>(wb + off); };
  e->embed = wp(off_embed);
  e->final_norm = wp(off_norm);
  e->lm_head = wp(off_lm);
  e->layers.resize(m.L);
  for (int l = 0; l < m.L; ++l) {
    e->layers[l] = LayerWeights{wp(lo[l].w_in), wp(lo[l].w_post), wp(lo[l].qkv_w), wp(lo[l].qkv_b),
                                wp(lo[l].o_w),  wp(lo[l].gu_w),   wp(lo[l].down_w)};
  }
  if (cudaMalloc(&e->d_layers, sizeof(LayerWeights) * m.L) != cudaSuccess) return fail("layer table allocation");
  cudaMemcpyAsync(e->d_layers, e->layers.data(), sizeof(LayerWeights) * m.L, cudaMemcpyHostToDevice, e->stream);

  // ---- caches, activations, control blocks: one allocation ----
  const size_t cache_elems = static_cast<size_t>(m.L) * m.NB * m.bs * m.nkv * m.d;
  size_t st = 0;
  auto take2 = [&](size_t bytes) {
    const size_t off = st;
    st = align_up(st + bytes, 256);
    return off;
  };
  const size_t o_k = take2(cache_elems * 2), o_v = take2(cache_elems * 2);
  const size_t o_cos = take2(static_cast<size_t>(m.C) * m.d * 2), o_sin = take2(static_cast<size_t>(m.C) * m.d * 2);
  const size_t o_h = take2(kBatch * H * 2), o_qkv = take2(static_cast<size_t>(kBatch) * m.Nqkv * 2);
  const size_t o_attn = take2(kBatch * H * 2), o_act = take2(static_cast<size_t>(kBatch) * m.I_pad * 2);
  const size_t o_av = take2(static_cast<size_t>(e->sms) * kBatch * 4);
  const size_t o_ai = take2(static_cast<size_t>(e->sms) * kBatch * 4);
  const size_t o_ab = take2(static_cast<size_t>(e->sms) * kBatch * 4);
  const size_t o_lg = take2(static_cast<size_t>(kMaxSteps) * kBatch * m.V * 4);
  const size_t o_trace = take2(kTraceSeries * kTraceMax * sizeof(uint64_t));
  const size_t o_io = take2(sizeof(EpochIO)), o_res = take2(sizeof(ResidentState));
  const size_t o_work = take2(sizeof(EpochWork)), o_sync = take2(sync_bytes(e->sms));
  if (cudaMalloc(&e->state, st) != cudaSuccess) return fail("state allocation");
  cudaMemsetAsync(e->state, 0, st, e->stream);
  uint8_t *sb = static_cast<uint8_t *>(e->state);
  e->key_cache = reinterpret_cast<bf16 *>(sb + o_k);
  e->value_cache = reinterpret_cast<bf16 *>(sb + o_v);
  e->rope_cos = reinterpret_cast<bf16 *>(sb + o_cos);
  e->rope_sin = reinterpret_cast<bf16 *>(sb + o_sin);
  e->h = reinterpret_cast<bf16 *>(sb + o_h);
  e->qkv = reinterpret_cast<bf16 *>(sb + o_qkv);
  e->attn = reinterpret_cast<bf16 *>(sb + o_attn);
  e->act = reinterpret_cast<bf16 *>(sb + o_act);
  e->partials = reinterpret_cast<uint64_t *>(sb + o_sync + sizeof(SyncState));
  e->arg_val = reinterpret_cast<float *>(sb + o_av);
  e->arg_idx = reinterpret_cast<int32_t *>(sb + o_ai);
  e->arg_bad = reinterpret_cast<int32_t *>(sb + o_ab);
  e->logits = reinterpret_cast<float *>(sb + o_lg);
  e->trace = reinterpret_cast<uint64_t *>(sb + o_trace);
  e->d_io = reinterpret_cast<EpochIO *>(sb + o_io);
  e->d_res = reinterpret_cast<ResidentState *>(sb + o_res);
  e->d_work = reinterpret_cast<EpochWork *>(sb + o_work);
  e->d_sync = reinterpret_cast<SyncState *>(sb + o_sync);
  if (cudaHostAlloc(reinterpret_cast<void **>(&e->h_io), sizeof(EpochIO), cudaHostAllocDefault) != cudaSuccess) {
    return fail("pinned host allocation");
  }
  if (e->tp_size > 1) {
    // the exchange block is its own allocation so that it can be exported by IPC
    if (cudaMalloc(reinterpret_cast<void **>(&e->xchg), sizeof(TpExchange)) != cudaSuccess ||
        cudaMalloc(reinterpret_cast<void **>(&e->d_peers), sizeof(TpExchange *) * kMaxTp) != cudaSuccess) {
      return fail("tensor-parallel exchange allocation");
    }
    cudaMemsetAsync(e->xchg, 0, sizeof(TpExchange), e->stream);
    cudaMemsetAsync(e->d_peers, 0, sizeof(TpExchange *) * kMaxTp, e->stream);
  }
  std::vector<uint16_t> cos_t, sin_t;
  default_rope(e, cos_t, sin_t);
  cudaMemcpyAsync(e->rope_cos, cos_t.data(), cos_t.size() * 2, cudaMemcpyHostToDevice, e->stream);
  cudaMemcpyAsync(e->rope_sin, sin_t.data(), sin_t.size() * 2, cudaMemcpyHostToDevice, e->stream);
  if (cudaStreamSynchronize(e->stream) != cudaSuccess) {
    *status = 3;
    return fail("initialising the resident state");
  }
  *status = 0;
  return e;
}

// ---- weight tensors by checkpoint name ---------------------------------------------------
struct TensorPlace {
  bf16 *base = nullptr;
  int64_t rows = 0, cols = 0;  // canonical shape
  bool tiled = false;          // false: a plain vector / row-major table at base + offset
  int32_t row_map = kRowOffset;
  int64_t offset = 0;          // destination row offset (plain: element offset)
  int64_t K = 0;               // packed columns of the tiled matrix
};

bool locate(Engine *e, const std::string &name, TensorPlace &tp) {
  const ModelDims &m = e->m;
  const int64_t H = m.H, kv = static_cast<int64_t>(m.nkv) * m.d;
  auto plain = [&](const bf16 *base, int64_t rows, int64_t cols, int64_t offset) {
    tp = TensorPlace{const_cast<bf16 *>(base), rows, cols, false, kRowOffset, offset, cols};
    return true;
  };
  auto tiled = [&](const bf16 *base, int64_t rows, int64_t cols, int32_t map, int64_t offset, int64_t K) {
    tp = TensorPlace{const_cast<bf16 *>(base), rows, cols, true, map, offset, K};
    return true;
  };
  if (name == "model.embed_tokens.weight") return plain(e->embed, m.V, H, 0);
  if (name == "model.norm.weight") return plain(e->final_norm, 1, H, 0);
  if (name == "lm_head.weight") return tiled(e->lm_head, m.Vl, H, kRowOffset, 0, H);
  const std::string prefix = "model.layers.";
  if (name.compare(0, prefix.size(), prefix) != 0) return false;
  const size_t dot = name.find('.', prefix.size());
  if (dot == std::string::npos) return false;
  const int layer = std::atoi(name.substr(prefix.size(), dot - prefix.size()).c_str());
  if (layer < 0 || layer >= m.L) return false;
  const std::string key = name.substr(dot + 1);
  const LayerWeights &lw = e->layers[layer];
  if (key == "input_layernorm.weight") return plain(lw.w_in, 1, H, 0);
  if (key == "post_attention_layernorm.weight") return plain(lw.w_post, 1, H, 0);
  const int64_t Hq = m.Hq;   // this rank's query rows (H without tensor parallelism)
  if (key == "self_attn.q_proj.weight") return tiled(lw.qkv_w, Hq, H, kRowOffset, 0, H);
  if (key == "self_attn.k_proj.weight") return tiled(lw.qkv_w, kv, H, kRowOffset, Hq, H);
  if (key == "self_attn.v_proj.weight") return tiled(lw.qkv_w, kv, H, kRowOffset, Hq + kv, H);
  if (key == "self_attn.q_proj.bias") return plain(lw.qkv_b, 1, Hq, 0);
  if (key == "self_attn.k_proj.bias") return plain(lw.qkv_b, 1, kv, Hq);
  if (key == "self_attn.v_proj.bias") return plain(lw.qkv_b, 1, kv, Hq + kv);
  if (key == "self_attn.o_proj.weight") return tiled(lw.o_w, H, Hq, kRowOffset, 0, m.Kq);
  if (key == "mlp.gate_proj.weight") return tiled(lw.gu_w, m.I, H, kRowGate, 0, H);
  if (key == "mlp.up_proj.weight") return tiled(lw.gu_w, m.I, H, kRowUp, 0, H);
  if (key == "mlp.down_proj.weight") return tiled(lw.down_w, H, m.I, kRowOffset, 0, m.I_pad);
  return false;
}

int32_t copy_tensor(Engine *e, const std::string &name, void *host, uint64_t bytes, bool to_device) {
  TensorPlace tp;
  if (!locate(e, name, tp)) return -1;
  if (bytes != static_cast<uint64_t>(tp.rows * tp.cols * 2)) return -1;
  cudaError_t err = cudaSuccess;
  if (!tp.tiled) {
    bf16 *dev = tp.base + tp.offset;
    err = to_device ? copy_sync(e, dev, host, bytes, cudaMemcpyHostToDevice)
                    : copy_sync(e, host, dev, bytes, cudaMemcpyDeviceToHost);
    return set_err(e, err, name.c_str());
  }
  void *staging = nullptr;
  err = cudaMalloc(&staging, bytes);
  if (err != cudaSuccess) return set_err(e, err, "weight staging");
  const int kc = pick_kc(static_cast<int>(tp.K));
  const int64_t count = tp.rows * tp.cols;
  const unsigned blocks = static_cast<unsigned>(std::min<int64_t>((count + 255) / 256, 148LL * 64));
  if (to_device) {
    err = copy_sync(e, staging, host, bytes, cudaMemcpyHostToDevice);
    if (err == cudaSuccess) {
      tile_copy_kernel<<<blocks, 256, 0, e->stream>>>(reinterpret_cast<uint16_t *>(tp.base),
                                                      static_cast<uint16_t *>(staging), tp.rows, tp.cols,
                                                      tp.row_map, tp.offset, tp.K, kc, 1);
      err = cudaGetLastError();
      if (err == cudaSuccess) err = cudaStreamSynchronize(e->stream);
    }
  } else {
    tile_copy_kernel<<<blocks, 256, 0, e->stream>>>(reinterpret_cast<uint16_t *>(tp.base),
                                                    static_cast<uint16_t *>(staging), tp.rows, tp.cols,
                                                    tp.row_map, tp.offset, tp.K, kc, 0);
    err = cudaGetLastError();
    if (err == cudaSuccess) err = cudaStreamSynchronize(e->stream);
    if (err == cudaSuccess) err = copy_sync(e, host, staging, bytes, cudaMemcpyDeviceToHost);
  }
  cudaFree(staging);
  return set_err(e, err, name.c_str());
}

// ---- batched device prefill ---------------------------------------------------------------------
int64_t import_payload_bytes(const Engine *e);

// ---- tensor-core GEMMs of the batched prefill (prefill_gemm.cuh) --------------------------
PFN_cuTensorMapEncodeTiled tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled fn = [] {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult found{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &found) != cudaSuccess ||
        found != cudaDriverEntryPointSuccess)
      ptr = nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled>(ptr);
  }();
  return fn;
}

// A tiled projection [N][K] (tiles of 16 rows x kc, stream order [row group][k
// tile]) as the 5-D tensor (element in a 128-byte segment, segment, row in
// tile, k tile, row group); a box is 8 row groups x 16 rows of one segment.
bool weight_map(CUtensorMap *map, const bf16 *W, int N, int K, int kc) {
  const PFN_cuTensorMapEncodeTiled encode = tensor_map_encoder();
  if (encode == nullptr) return false;
  const cuuint64_t dims[5] = {64, static_cast<cuuint64_t>(kc / 64), 16, static_cast<cuuint64_t>(K / kc),
                              static_cast<cuuint64_t>(N / 16)};
  const cuuint64_t strides[4] = {128, static_cast<cuuint64_t>(kc) * 2, static_cast<cuuint64_t>(kc) * 32,
                                 static_cast<cuuint64_t>(K / kc) * kc * 32};
  const cuuint32_t box[5] = {64, 1, 16, 1, tcgemm::kM / 16};
  const cuuint32_t elem[5] = {1, 1, 1, 1, 1};
  return encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 5, const_cast<bf16 *>(W), dims, strides, box, elem,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Row-major activations [T][width] (row pitch `pitch` elements) in boxes of
// 64 columns x `rows` tokens with the 128-byte swizzle; out-of-range reads zero.
bool activation_map(CUtensorMap *map, const bf16 *X, int T, int width, int pitch, int rows) {
  const PFN_cuTensorMapEncodeTiled encode = tensor_map_encoder();
  if (encode == nullptr) return false;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(width), static_cast<cuuint64_t>(T)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(pitch) * 2};
  const cuuint32_t box[2] = {64, static_cast<cuuint32_t>(rows)};
  const cuuint32_t elem[2] = {1, 1};
  return encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<bf16 *>(X), dims, strides, box, elem,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The GEMM's fp32 partial sums [split][T][N] as a 3-D tensor (row, token,
// split) for its tensor stores: boxes of 32 rows x 8 tokens.
bool partial_map(CUtensorMap *map, float *P, int N, int T, int nsplit) {
  const PFN_cuTensorMapEncodeTiled encode = tensor_map_encoder();
  if (encode == nullptr) return false;
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(N), static_cast<cuuint64_t>(T),
                              static_cast<cuuint64_t>(nsplit)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(N) * 4, static_cast<cuuint64_t>(N) * T * 4};
  const cuuint32_t box[3] = {32, static_cast<cuuint32_t>(tcgemm::kStoreTokens), 1};
  const cuuint32_t elem[3] = {1, 1, 1};
  return encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, P, dims, strides, box, elem, CU_TENSOR_MAP_INTERLEAVE_NONE,
                CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// CTA pairs of the GEMM that can be resident at once (one CTA per SM).  The
// first call raises the kernel's shared-memory limit.
int gemm_pairs(Engine *e) {
  PrefillState *ps = e->prefill;
  if (ps->gemm_pairs > 0) return ps->gemm_pairs;
  if (!ps->gemm_attr) {
    if (cudaFuncSetAttribute(tcgemm::gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(tcgemm::smem_bytes())) != cudaSuccess) {
      cudaGetLastError();
      return e->sms / 2;   // the launch reports the failure
    }
    ps->gemm_attr = true;
  }
  cudaLaunchConfig_t cfg{};
  cudaLaunchAttribute attr{};
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = 2;
  attr.val.clusterDim.y = 1;
  attr.val.clusterDim.z = 1;
  cfg.gridDim = dim3(2 * (e->sms / 2));
  cfg.blockDim = dim3(tcgemm::kThreads);
  cfg.dynamicSmemBytes = tcgemm::smem_bytes();
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  int clusters = 0;
  if (cudaOccupancyMaxActiveClusters(&clusters, tcgemm::gemm_kernel, &cfg) != cudaSuccess || clusters <= 0) {
    cudaGetLastError();
    clusters = e->sms / 2;
  }
  ps->gemm_pairs = std::min(clusters, e->sms / 2);
  return ps->gemm_pairs;
}

// Launches a prefill kernel as a programmatic dependent of the previous one in
// the stream (when enabled): it may begin while that one drains and waits for
// it inside (prefill::chain_enter).
template <typename... Params, typename... Actual>
void chain_launch(Engine *e, dim3 grid, dim3 block, size_t smem, void (*kernel)(Params...), Actual &&...args) {
  cudaLaunchConfig_t cfg{};
  cudaLaunchAttribute attr{};
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = e->prefill->chain ? 1 : 0;
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = e->stream;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, kernel, std::forward<Actual>(args)...);   // errors surface at the stream check
}

// How a projection is tiled: tokens per pair tile and k-range splits.
struct GemmPlan {
  int ttile = 512, ttiles = 1, nsplit = 1;
};

// k-range splits for `tiles` pair tiles of `chunks` k chunks: tiles x splits
// run in waves over the resident pairs; the split count minimises waves x
// chunks per split, plus two chunks' worth per split for the partial sums it
// adds.
int gemm_splits(Engine *e, int tiles, int chunks) {
  const int pairs = gemm_pairs(e);
  int best = 1;
  int64_t best_cost = INT64_MAX;
  for (int sp = 1; sp <= std::min(chunks, prefill::kMaxSplits); ++sp) {
    const int64_t waves = (static_cast<int64_t>(tiles) * sp + pairs - 1) / pairs;
    const int64_t cost = waves * ((chunks + sp - 1) / sp) + 2 * sp;
    if (cost < best_cost) {
      best_cost = cost;
      best = sp;
    }
  }
  return best;
}

// All tokens in one tile (W read once per tile: the copies from L2 set the
// pace, and 128-token tiles measured slower for QKV and O), k split where
// the row tiles alone do not fill the pairs.  `narrow_tile` (0: all tokens)
// caps the token tile of the split projections.
GemmPlan gemm_plan(Engine *e, int N, int K, int T, bool splittable = true) {
  GemmPlan p;
  p.ttile = T <= 128 ? 128 : T <= 256 ? 256 : 512;
  if (splittable && e->prefill->narrow_tile > 0) p.ttile = std::min(p.ttile, e->prefill->narrow_tile);
  p.ttiles = (T + p.ttile - 1) / p.ttile;
  p.nsplit = splittable ? gemm_splits(e, (N + tcgemm::kRows - 1) / tcgemm::kRows * p.ttiles, K / tcgemm::kKChunk) : 1;
  if (splittable && e->prefill->force_split > 0) p.nsplit = std::min(e->prefill->force_split, prefill::kMaxSplits);
  return p;
}

// Y = X . W^T on the tensor cores.  mode 0: fp32 partials [nsplit][T][N] into
// ps->acc; mode 1 (the interleaved gate/up projection): the SwiGLU activation
// [T][N / 2] into `out`; mode 2 (no k splits): bf16 [T][N] into `out`.
// Returns false, with the reason in last_error, when a tensor map cannot be
// made or the launch fails.
bool prefill_gemm(Engine *e, const bf16 *W, int N, int K, const bf16 *X, int T, int x_width, int mode,
                  const GemmPlan &plan, bf16 *out) {
  PrefillState *ps = e->prefill;
  tcgemm::Args a{};
  a.T = T;
  a.N = N;
  a.chunks = K / tcgemm::kKChunk;
  a.kc = pick_kc(K);
  a.nsplit = plan.nsplit;
  a.mode = mode;
  a.ttile = plan.ttile;
  a.ttiles = plan.ttiles;
  a.tsub = plan.ttile > tcgemm::kSub ? 2 : 1;
  a.xrows = std::min(plan.ttile / 2, tcgemm::kSub / 2);
  a.stages = std::min<int>(tcgemm::kMaxStages, tcgemm::kRingBytes / tcgemm::stage_bytes(a.tsub, a.xrows));
  if (ps->stage_cap >= 2) a.stages = std::min(a.stages, ps->stage_cap);
  a.tiles = (N + tcgemm::kRows - 1) / tcgemm::kRows * plan.ttiles * plan.nsplit;
  a.partials = ps->acc;
  a.out = out;
  a.out_stride = mode == 1 ? N / 2 : N;
  a.error = ps->error;
  a.w_evict_first = ps->w_evict_first ? 1 : 0;
  a.p_evict_last = ps->p_evict_last ? 1 : 0;
  a.trace = nullptr;
  const int pairs_now = gemm_pairs(e);
  if (ps->trace != nullptr && ps->trace_calls < kTraceLaunches) {
    ps->trace_grid[ps->trace_calls] = 2 * std::min(a.tiles, pairs_now);
    a.trace = ps->trace + static_cast<size_t>(ps->trace_calls++) * e->sms * tcgemm::kTraceMarks;
  }
  CUtensorMap wmap, xmap, pmap;
  // modes 1 and 2 store no partial sums: a small placeholder map
  const bool parts = mode == 0;
  if (!weight_map(&wmap, W, N, K, a.kc) || !activation_map(&xmap, X, T, x_width, x_width, a.xrows) ||
      !partial_map(&pmap, ps->acc, parts ? N : 32, parts ? T : 8, parts ? plan.nsplit : 1)) {
    e->last_error = "prefill: a GEMM tensor map could not be encoded";
    return false;
  }
  const size_t smem = tcgemm::smem_bytes();
  const int pairs = gemm_pairs(e);
  if (!ps->gemm_attr) {
    e->last_error = "prefill: the GEMM's shared-memory size (" + std::to_string(smem) + " bytes) was refused";
    return false;
  }
  cudaLaunchConfig_t cfg{};
  cudaLaunchAttribute attr[2]{};
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = ps->chain ? 1 : 0;
  cfg.gridDim = dim3(2 * std::min(a.tiles, pairs));
  cfg.blockDim = dim3(tcgemm::kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = e->stream;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  const cudaError_t err = cudaLaunchKernelEx(&cfg, tcgemm::gemm_kernel, wmap, xmap, pmap, a);
  if (err != cudaSuccess) {
    e->last_error = std::string("prefill: GEMM launch: ") + cudaGetErrorString(err);
    cudaGetLastError();
    return false;
  }
  return true;
}

// Profiling summary of the traced GEMM launches (stderr), in µs after the
// moment the launch's predecessor had completed (the earliest "predecessor
// complete" mark): per launch the CTA medians of entry, first load issued,
// first stage landed and last MMA committed (leaders), first accumulators
// ready, epilogue done, and the median and last exit.
void print_gemm_trace(Engine *e) {
  PrefillState *ps = e->prefill;
  const int per = e->sms * tcgemm::kTraceMarks;
  std::vector<uint64_t> h(static_cast<size_t>(kTraceLaunches) * per);
  if (copy_sync(e, h.data(), ps->trace, h.size() * 8, cudaMemcpyDeviceToHost) != cudaSuccess) return;
  static const char *names[kTraceLaunches] = {"qkv", "o", "gate_up", "down", "qkv", "o", "gate_up", "down"};
  std::fprintf(stderr, "prefill GEMM trace (us after predecessor done): launch grid | entry first_load first_stage "
                       "last_mma(leaders) first_acc epi_done | exit_median exit_last\n");
  for (int i = 0; i < ps->trace_calls; ++i) {
    const uint64_t *t = h.data() + static_cast<size_t>(i) * per;
    const int grid = ps->trace_grid[i];
    uint64_t base = UINT64_MAX;
    for (int c = 0; c < grid; ++c)
      if (t[c * tcgemm::kTraceMarks + 1] != 0) base = std::min(base, t[c * tcgemm::kTraceMarks + 1]);
    if (base == UINT64_MAX) continue;
    auto median = [&](int mark, bool leaders_only, bool last) {
      std::vector<double> v;
      for (int c = 0; c < grid; ++c) {
        if (leaders_only && (c & 1)) continue;
        const uint64_t x = t[c * tcgemm::kTraceMarks + mark];
        if (x != 0) v.push_back((static_cast<double>(x) - static_cast<double>(base)) / 1e3);
      }
      if (v.empty()) return 0.0;
      std::sort(v.begin(), v.end());
      return last ? v.back() : v[v.size() / 2];
    };
    std::fprintf(stderr, "  L%d %-8s %4d | %7.2f %7.2f %7.2f %7.2f %7.2f %7.2f | %7.2f %7.2f\n", i / 4, names[i], grid,
                 median(0, false, false), median(2, false, false), median(3, true, false), median(4, true, false),
                 median(5, false, false), median(6, false, false), median(7, false, false), median(7, false, true));
  }
}

// Frees the prefill buffers, whole or partly built; cudaFree waits for the
// work queued on them.
void prefill_release(Engine *e) {
  PrefillState *ps = e->prefill;
  if (ps == nullptr) return;
  cudaFree(ps->work);
  if (ps->trace != nullptr) cudaFree(ps->trace);
  delete ps;
  e->prefill = nullptr;
}

// Buffers for kBatch * block_size tokens.  A failure leaves the state partly
// built; the caller releases it, so the next call starts over instead of using it.
int32_t prefill_prepare(Engine *e) {
  if (e->prefill != nullptr) return 0;
  const ModelDims &m = e->m;
  const int64_t H = m.H, Hq = m.Hq, I = m.I, N = m.Nqkv;
  auto *ps = new PrefillState();
  e->prefill = ps;
  if (const char *env = std::getenv("CRUISE_PREFILL_PDL")) ps->chain = std::atoi(env) != 0;
  if (const char *env = std::getenv("CRUISE_PREFILL_TTILE")) {
    const int v = std::atoi(env);
    ps->narrow_tile = v == 128 || v == 256 || v == 512 ? v : 0;
  }
  if (const char *env = std::getenv("CRUISE_PREFILL_SPLIT")) ps->force_split = std::max(0, std::atoi(env));
  if (const char *env = std::getenv("CRUISE_PREFILL_WHINT")) ps->w_evict_first = std::atoi(env) != 0;
  if (const char *env = std::getenv("CRUISE_PREFILL_STAGES")) ps->stage_cap = std::max(0, std::atoi(env));
  if (const char *env = std::getenv("CRUISE_PREFILL_PHINT")) ps->p_evict_last = std::atoi(env) != 0;
  if (tensor_map_encoder() == nullptr) {
    e->last_error = "prefill: the driver has no cuTensorMapEncodeTiled";
    return -2;
  }
  // activations for every prompt token of a cohort: at most block_size per row
  const int T = kBatch * m.bs;
  ps->max_tokens = T;
  // the most fp32 partial sums (splits x outputs x tokens) of QKV, O and down
  // at any token count: the plans change only where a 128-token tile fills
  // up, so each range's largest count stands for it
  int64_t parts = 0;
  for (int t = 128;; t += 128) {
    const int tt = std::min(T, t);
    const int64_t sq = gemm_plan(e, m.Nqkv, m.H, tt).nsplit, so = gemm_plan(e, m.H, m.Hq, tt).nsplit;
    const int64_t sd = gemm_plan(e, m.H, m.I_pad, tt).nsplit;
    parts = std::max(parts, std::max(sq * N, std::max(so, sd) * H) * tt);
    if (tt == T) break;
  }
  size_t bytes = 0;
  auto take = [&](size_t n) { const size_t off = bytes; bytes = align_up(bytes + n, 1024); return off; };
  const size_t o_h = take(T * H * 2), o_x = take(T * H * 2), o_q = take(T * Hq * 2), o_attn = take(T * Hq * 2);
  const size_t o_act = take(T * I * 2), o_y = take(T * H * 2), o_acc = take(parts * 4), o_tok = take(T * 8),
               o_row = take(T * 4),
               o_pos = take(T * 4), o_err = take(4);
  cudaError_t err = cudaMalloc(&ps->work, bytes);
  if (err != cudaSuccess) return set_err(e, err, "prefill buffers");
  uint8_t *b = static_cast<uint8_t *>(ps->work);
  ps->h = reinterpret_cast<bf16 *>(b + o_h);
  ps->x = reinterpret_cast<bf16 *>(b + o_x);
  ps->q = reinterpret_cast<bf16 *>(b + o_q);
  ps->attn = reinterpret_cast<bf16 *>(b + o_attn);
  ps->act = reinterpret_cast<bf16 *>(b + o_act);
  ps->y = reinterpret_cast<bf16 *>(b + o_y);
  ps->acc = reinterpret_cast<float *>(b + o_acc);
  ps->tok = reinterpret_cast<int64_t *>(b + o_tok);
  ps->row = reinterpret_cast<int32_t *>(b + o_row);
  ps->pos = reinterpret_cast<int32_t *>(b + o_pos);
  ps->error = reinterpret_cast<uint32_t *>(b + o_err);
  err = cudaMemsetAsync(ps->work, 0, bytes, e->stream);
  if (err == cudaSuccess) {
    const char *env = std::getenv("CRUISE_PREFILL_TRACE");
    if (env != nullptr && std::atoi(env) != 0)
      err = cudaMalloc(&ps->trace, sizeof(uint64_t) * kTraceLaunches * e->sms * tcgemm::kTraceMarks);
  }
  if (err == cudaSuccess) err = cudaStreamSynchronize(e->stream);
  return set_err(e, err, "prefill preparation");
}

// The K/V of prompt tokens 0..len-2 of every row (the decode epoch starts at
// position len-1) into the import staging buffer, layer by layer for all tokens.
int32_t prefill_run(Engine *e, const int64_t *tokens, const int32_t *lens, int32_t stride) {
  const ModelDims &m = e->m;
  if (e->tp_size > 1 || m.Kq != m.Hq) {
    e->last_error = "cruise_epoch_prefill: single-GPU engines only (no tensor parallelism)";
    return -4;
  }
  if (m.bs > prefill::kMaxKeys || (m.d != 64 && m.d != 128) || m.nq / m.nkv * prefill::kAttnChunk > prefill::kMaxKeys ||
      m.I % 8 != 0 || m.H % 8 != 0 || m.H > 8 * prefill::kNormThreads * prefill::kNormChunks) {
    e->last_error = "cruise_epoch_prefill: needs block size <= 128, head size 64 or 128, <= 8 query heads per KV head,"
                    " an intermediate size divisible by 8 and a hidden size divisible by 8, at most 8192";
    return -1;
  }
  std::vector<int64_t> tok;
  std::vector<int32_t> row, pos;
  for (int r = 0; r < kBatch; ++r) {
    if (lens[r] < 0 || lens[r] > m.bs || lens[r] > stride) {
      e->last_error = "cruise_epoch_prefill: prompt lengths must lie in [0, block_size]";
      return -1;
    }
    for (int t = 0; t + 1 < lens[r]; ++t) {
      const int64_t id = tokens[static_cast<int64_t>(r) * stride + t];
      if (id < 0 || id >= m.V) {
        e->last_error = "cruise_epoch_prefill: token id outside the vocabulary";
        return -1;
      }
      tok.push_back(id);
      row.push_back(r);
      pos.push_back(t);
    }
  }
  int32_t rc = prefill_prepare(e);
  if (rc != 0) {
    prefill_release(e);
    return rc;
  }
  PrefillState *ps = e->prefill;
  const size_t payload_bytes = static_cast<size_t>(import_payload_bytes(e));
  cudaError_t err = cudaSuccess;
  if (e->d_payload == nullptr) {
    err = cudaMalloc(&e->d_payload, payload_bytes);
    if (err != cudaSuccess) return set_err(e, err, "import staging");
    e->payload_bytes = payload_bytes;
  }
  err = cudaMemsetAsync(e->d_payload, 0, payload_bytes, e->stream);
  const int T = static_cast<int>(tok.size());
  if (err == cudaSuccess && T > 0) {
    err = cudaMemcpyAsync(ps->tok, tok.data(), T * 8, cudaMemcpyHostToDevice, e->stream);
    if (err == cudaSuccess) err = cudaMemcpyAsync(ps->row, row.data(), T * 4, cudaMemcpyHostToDevice, e->stream);
    if (err == cudaSuccess) err = cudaMemcpyAsync(ps->pos, pos.data(), T * 4, cudaMemcpyHostToDevice, e->stream);
  }
  if (err != cudaSuccess) return set_err(e, err, "prefill inputs");
  bf16 *payload = reinterpret_cast<bf16 *>(e->d_payload);
  const int H = m.H, I = m.I;
  // attention: one CTA per (16-position chunk, KV head, row) over the packed tokens
  prefill::RowSpans spans{};
  int longest = 0;
  for (int r = 0, start = 0; r < kBatch; ++r) {
    spans.start[r] = start;
    spans.count[r] = std::max(lens[r] - 1, 0);
    start += spans.count[r];
    longest = std::max(longest, spans.count[r]);
  }
  const dim3 attn_grid((longest + prefill::kAttnChunk - 1) / prefill::kAttnChunk, m.nkv, kBatch);
  const size_t attn_smem = prefill::attention_smem_bytes(m.bs, m.d, m.nq / m.nkv);
  auto *attention = m.d == 128 ? prefill::causal_attention_mma<128> : prefill::causal_attention_mma<64>;
  if (T > 0 && cudaFuncSetAttribute(attention, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(attn_smem)) != cudaSuccess)
    return set_err(e, cudaGetLastError(), "prefill attention shared memory");
  bool gemm_ok = true;
  if (T > 0) {
    const GemmPlan pq = gemm_plan(e, m.Nqkv, H, T), po = gemm_plan(e, H, m.Hq, T);
    const GemmPlan pg = gemm_plan(e, 2 * I, H, T, false), pd = gemm_plan(e, H, m.I_pad, T);
    // qkv_rope_store: one unit (a rotation pair of q or k elements, or two v elements) per thread
    const unsigned rope_rows = static_cast<unsigned>(((m.nq + m.nkv) * (m.d / 4) + m.nkv * m.d / 2 + 255) / 256);
    const unsigned parts_threads = static_cast<unsigned>(prefill::parts_norm_threads(H));
    err = cudaMemsetAsync(ps->error, 0, 4, e->stream);
    ps->trace_calls = 0;
    if (err == cudaSuccess && ps->trace != nullptr)
      err = cudaMemsetAsync(ps->trace, 0, sizeof(uint64_t) * kTraceLaunches * e->sms * tcgemm::kTraceMarks,
                            e->stream);
    if (err != cudaSuccess) return set_err(e, err, "prefill error word");
    prefill::embed_rows<<<T, 128, 0, e->stream>>>(e->embed, ps->tok, ps->h, H);
    chain_launch(e, T, 256, 0, prefill::rms_norm_rows, ps->h, e->layers[0].w_in, ps->x, H, m.eps);
    for (int l = 0; l < m.L && gemm_ok; ++l) {
      // x holds rms_norm(h) * w_in of this layer
      const LayerWeights &lw = e->layers[l];
      gemm_ok &= prefill_gemm(e, lw.qkv_w, m.Nqkv, H, ps->x, T, H, 0, pq, nullptr);
      chain_launch(e, dim3(T, rope_rows), 256, 0, prefill::qkv_rope_store, ps->acc, pq.nsplit, T, lw.qkv_b,
                   e->rope_cos, e->rope_sin, ps->row, ps->pos, ps->q, payload, l, m.L, m.nq, m.nkv, m.d, m.bs);
      // the last layer's K/V are its only output the payload holds: its
      // attention, O projection and MLP would feed no later layer
      if (l == m.L - 1) break;
      chain_launch(e, attn_grid, prefill::kAttnWarps * 32, attn_smem, attention, ps->q, payload, spans, ps->attn, l,
                   m.L, m.nq, m.nkv, m.bs, m.sqrt_d);
      if (po.nsplit == 1) {   // bf16 out of the GEMM: the decoder's materialize(mm_t(attn, Wo))
        gemm_ok &= prefill_gemm(e, lw.o_w, H, m.Hq, ps->attn, T, m.Hq, 2, po, ps->y);
        chain_launch(e, T, prefill::kNormThreads, 0, prefill::residual_rms_norm, ps->y, ps->h, lw.w_post, ps->x, H,
                     m.eps);
      } else {
        gemm_ok &= prefill_gemm(e, lw.o_w, H, m.Hq, ps->attn, T, m.Hq, 0, po, nullptr);
        chain_launch(e, T, parts_threads, 0, prefill::residual_rms_norm_parts, ps->acc, po.nsplit, T, ps->h,
                     lw.w_post, ps->x, H, m.eps);
      }
      // gate/up with the SwiGLU in its epilogue (needs whole sums: no k split): the activation [T][I]
      gemm_ok &= prefill_gemm(e, lw.gu_w, 2 * I, H, ps->x, T, H, 1, pg, ps->act);
      gemm_ok &= prefill_gemm(e, lw.down_w, H, m.I_pad, ps->act, T, I, 0, pd, nullptr);
      chain_launch(e, T, parts_threads, 0, prefill::residual_rms_norm_parts, ps->acc, pd.nsplit, T, ps->h,
                   e->layers[l + 1].w_in, ps->x, H, m.eps);
    }
  }
  if (!gemm_ok) return -2;   // prefill_gemm left the reason in last_error
  err = cudaGetLastError();
  if (err == cudaSuccess) err = cudaStreamSynchronize(e->stream);
  if (err != cudaSuccess) return set_err(e, err, "prefill");
  if (T > 0) {
    uint32_t site = 0;
    err = copy_sync(e, &site, ps->error, 4, cudaMemcpyDeviceToHost);
    if (err != cudaSuccess) return set_err(e, err, "prefill error word");
    if (site != 0) {
      e->last_error = "prefill: a tensor-core GEMM wait gave up (site " + std::to_string(site) + ")";
      return -2;
    }
    if (ps->trace != nullptr) print_gemm_trace(e);
  }
  e->payload_ready = true;
  return 0;
}

int32_t synth_all(Engine *e, uint64_t seed, double stddev) {
  const ModelDims &m = e->m;
  const double sigma = 2.0 * std::sqrt(4.0 * (65536.0 * 65536.0 - 1.0) / 12.0);
  const float scale = static_cast<float>(stddev / sigma);
  const int64_t H = m.H, kv = static_cast<int64_t>(m.nkv) * m.d;
  auto launch = [&](bf16 *dst, int64_t count, SynthMap map) {
    const int threads = 256;
    const int64_t blocks = std::min<int64_t>((count + threads - 1) / threads, 148LL * 64);
    synth_kernel<<<static_cast<unsigned>(blocks), threads, 0, e->stream>>>(
        reinterpret_cast<uint16_t *>(dst), count, map, seed, scale);
  };
  auto plain = [&](int id) { SynthMap s{}; s.mode = kPlain; s.ids[0] = id; return s; };
  auto tile = [&](SynthMap s, int64_t K) { s.tiled = 1; s.dst_cols = K; s.kc = pick_kc(static_cast<int>(K)); return s; };
  const int L = m.L;
  launch(e->embed, static_cast<int64_t>(m.V) * H, plain(0));
  for (int l = 0; l < L; ++l) {
    const int base = 1 + kLayerTensors * l;
    const LayerWeights &lw = e->layers[l];
    launch(const_cast<bf16 *>(lw.w_in), H, plain(base + 0));
    launch(const_cast<bf16 *>(lw.w_post), H, plain(base + 1));
    SynthMap q{};
    q.mode = kQkvRows; q.ids[0] = base + 2; q.ids[1] = base + 4; q.ids[2] = base + 6;
    q.cols = H; q.rows0 = m.Hq; q.rows1 = kv;
    q.off0 = static_cast<int64_t>(m.q0) * m.d; q.off1 = static_cast<int64_t>(m.kv0) * m.d;
    SynthMap qb = q;
    qb.ids[0] = base + 3; qb.ids[1] = base + 5; qb.ids[2] = base + 7; qb.cols = 1;
    launch(const_cast<bf16 *>(lw.qkv_w), static_cast<int64_t>(m.Nqkv) * H, tile(q, H));
    launch(const_cast<bf16 *>(lw.qkv_b), m.Nqkv, qb);
    SynthMap o{};
    // this rank's Hq columns of the canonical [H][H] tensor, zero up to Kq
    o.mode = kDownPad; o.ids[0] = base + 8; o.cols = H; o.rows0 = m.Hq; o.dst_cols = m.Kq;
    o.off0 = static_cast<int64_t>(m.q0) * m.d;
    launch(const_cast<bf16 *>(lw.o_w), H * m.Kq, tile(o, m.Kq));
    SynthMap gu{};
    gu.mode = kGateUp; gu.ids[0] = base + 9; gu.ids[1] = base + 10; gu.cols = H;
    gu.off0 = static_cast<int64_t>(e->tp_rank) * m.I;
    launch(const_cast<bf16 *>(lw.gu_w), 2LL * m.I * H, tile(gu, H));
    SynthMap dn{};
    dn.mode = kDownPad; dn.ids[0] = base + 11; dn.cols = e->cfg.intermediate; dn.rows0 = m.I;
    dn.off0 = static_cast<int64_t>(e->tp_rank) * m.I;
    dn = tile(dn, m.I_pad);
    launch(const_cast<bf16 *>(lw.down_w), H * m.I_pad, dn);
  }
  launch(e->final_norm, H, plain(1 + kLayerTensors * L));
  SynthMap lm{};
  lm.mode = kRowsPad; lm.ids[0] = 2 + kLayerTensors * L; lm.cols = H; lm.rows0 = m.Vl; lm.off0 = m.v0;
  launch(e->lm_head, static_cast<int64_t>(m.V_pad) * H, tile(lm, H));
  cudaError_t err = cudaGetLastError();
  if (err == cudaSuccess) err = cudaStreamSynchronize(e->stream);
  return set_err(e, err, "synthetic weights");
}

int64_t import_payload_bytes(const Engine *e) {
  return 2LL * e->m.L * kBatch * e->m.bs * e->m.nkv_all * e->m.d * 2;   // every KV head of the model
}

// Launch parameters of a regular (engine-allocated) launch: the model, the
// resident caches and state, the engine's scratch, the launch geometry.
EpochParams engine_params(const Engine *e) {
  EpochParams p{};
  p.m = e->m;
  p.layers = e->d_layers;
  p.embed = e->embed;
  p.final_norm = e->final_norm;
  p.lm_head = e->lm_head;
  p.rope_cos = e->rope_cos;
  p.rope_sin = e->rope_sin;
  p.key_cache = e->key_cache;
  p.value_cache = e->value_cache;
  p.h = e->h;
  p.qkv = e->qkv;
  p.attn = e->attn;
  p.act = e->act;
  p.partials = e->partials;
  p.arg_val = e->arg_val;
  p.arg_idx = e->arg_idx;
  p.arg_bad = e->arg_bad;
  p.io = e->d_io;
  p.res = e->d_res;
  p.work = e->d_work;
  p.sync = e->d_sync;
  p.grid = e->sms;
  p.stages = e->stages;
  p.xs_stride = e->xs_stride;
  p.down_xglobal = e->down_xglobal;
  p.o_xglobal = e->o_xglobal;
  p.trace = e->trace_on ? e->trace : nullptr;
  p.trace_cta = e->trace_cta_on ? e->trace_cta : nullptr;
  p.l2_ahead = e->l2_ahead;
  p.l2_hints = e->l2_hints;
  p.mode = kModeEpoch;
  return p;
}

// One epoch: H2D of the 8 inputs (+ optional import payload), one cooperative
// launch, D2H of the 2 outputs.
int32_t run_epoch(Engine *e, const int64_t *token, const int64_t *position, const int32_t *seq_len,
                  const int32_t *slot, const int32_t *active, const int32_t *block_table,
                  const uint8_t *tiling, const int32_t *control, const void *payload,
                  uint64_t payload_bytes, int64_t *history, int32_t *control_out, float *logits_out,
                  const int64_t *forced = nullptr, bool payload_on_device = false) {
  cudaSetDevice(e->device);
  EpochIO *io = e->h_io;
  std::memset(io, 0, sizeof(EpochIO));
  std::memcpy(io->token, token, sizeof(io->token));
  std::memcpy(io->position, position, sizeof(io->position));
  std::memcpy(io->seq_len, seq_len, sizeof(io->seq_len));
  std::memcpy(io->slot, slot, sizeof(io->slot));
  std::memcpy(io->active, active, sizeof(io->active));
  std::memcpy(io->block_table, block_table, sizeof(int32_t) * kBatch * e->m.bpr);
  std::memcpy(io->control, control, sizeof(io->control));
  if (tiling != nullptr) std::memcpy(io->tiling, tiling, kTilingBytes);
  if (forced != nullptr) {
    io->use_forced = 1;
    std::memcpy(io->forced, forced, sizeof(io->forced));
  }
  const bool importing = (control[2 + kBatch] & kImportFlag) != 0;
  cudaError_t err = cudaSuccess;
  if (importing && payload == nullptr && payload_bytes == 0) {
    // the cohort cruise_epoch_prefill left in the device staging buffer
    if (!e->payload_ready) {
      e->last_error = "import without a payload and no prefilled cohort on the device";
      return -1;
    }
    payload = e->d_payload;
    payload_bytes = static_cast<uint64_t>(import_payload_bytes(e));
    payload_on_device = true;
    e->payload_ready = false;
  }
  if (importing) {
    if (payload == nullptr || payload_bytes != static_cast<uint64_t>(import_payload_bytes(e))) return -1;
    if (!payload_on_device) {
      if (e->d_payload == nullptr) {
        err = cudaMalloc(&e->d_payload, payload_bytes);
        if (err != cudaSuccess) return set_err(e, err, "import staging");
        e->payload_bytes = payload_bytes;
      }
      err = cudaMemcpyAsync(e->d_payload, payload, payload_bytes, cudaMemcpyHostToDevice, e->stream);
      if (err != cudaSuccess) return set_err(e, err, "import payload copy");
      e->payload_ready = false;   // a prefilled cohort in the staging buffer is overwritten
    }
  }
  const size_t in_bytes = offsetof(EpochIO, history);
  err = cudaMemcpyAsync(e->d_io, io, in_bytes, cudaMemcpyHostToDevice, e->stream);
  if (err == cudaSuccess) err = cudaMemsetAsync(e->d_sync, 0, sync_bytes(e->sms), e->stream);
  if (err != cudaSuccess) return set_err(e, err, "epoch inputs");

  EpochParams p = engine_params(e);
  p.logits = logits_out != nullptr ? e->logits : nullptr;
  p.import_payload = payload_on_device ? static_cast<const uint8_t *>(payload) : e->d_payload;
  if (e->trace_on) cudaMemsetAsync(e->trace, 0, kTraceSeries * kTraceMax * sizeof(uint64_t), e->stream);
  if (e->trace_cta_on)
    cudaMemsetAsync(e->trace_cta, 0, static_cast<size_t>(kTraceMax) * e->sms * kTraceCtaWords * sizeof(uint32_t), e->stream);
  // every device-side wait gives up after 2 s; under tensor parallelism after
  // 20 s by default (CRUISE_TP_TIMEOUT_MS at creation), since a rank's first
  // wait also covers the other ranks' launch skew
  p.timeout_ns = e->tp_size > 1 ? e->tp_timeout_ns : 2000000000ull;
  p.tp_size = e->tp_size;
  p.tp_rank = e->tp_rank;
  if (e->tp_size > 1) {
    if (!e->tp_connected) {
      e->last_error = "tensor-parallel engine used before cruise_epoch_tp_connect";
      return -5;
    }
    p.tp_peer = e->d_peers;
    p.tp_local = e->xchg;
  }
  // exchange sequence numbers grow across launches (every rank launches the
  // same epochs); a launch uses at most 8 x 142 of its 65,536
  p.launch_id = ++e->launches;
  p.tp_seq_base = p.launch_id << 16;
  p.stream = e->stream_on ? e->d_stream : nullptr;
  void *args[] = {&p};
  cudaEventRecord(e->ev0, e->stream);
  err = cudaLaunchCooperativeKernel(reinterpret_cast<const void *>(resident_epoch_kernel), dim3(e->sms),
                                    dim3(kThreads), args, e->smem, e->stream);
  cudaEventRecord(e->ev1, e->stream);
  if (err != cudaSuccess) return set_err(e, err, "epoch launch");
  err = cudaMemcpyAsync(&io->history, &e->d_io->history,
                        sizeof(EpochIO) - offsetof(EpochIO, history), cudaMemcpyDeviceToHost, e->stream);
  if (err == cudaSuccess && logits_out != nullptr) {
    err = cudaMemcpyAsync(logits_out, e->logits, sizeof(float) * kMaxSteps * kBatch * e->m.V,
                          cudaMemcpyDeviceToHost, e->stream);
  }
  if (err == cudaSuccess) err = cudaStreamSynchronize(e->stream);
  if (err != cudaSuccess) return set_err(e, err, "epoch completion");
  cudaEventElapsedTime(&e->last_ms, e->ev0, e->ev1);
  e->last_launches = 1;
  std::memcpy(history, io->history, sizeof(io->history));
  std::memcpy(control_out, io->control_out, sizeof(io->control_out));
  if (control_out[3] == kModelError) {
    // which device-side wait gave up (sites: 1-4 prologue barriers, 100+phase
    // grid barriers, 300 tensor-parallel partials, 401 tensor-parallel argmax,
    // 900/1001-1004 pipeline waits)
    uint32_t words[2] = {0, 0};
    if (copy_sync(e, words, &e->d_sync->error, sizeof(words), cudaMemcpyDeviceToHost) == cudaSuccess && words[0])
      e->last_error = "epoch ended by a device-side wait that gave up (site " + std::to_string(words[1]) + ")";
  }
  return 0;
}

// One decoder call of the 9-input / 4-output decoder ABI (config/graph_config.json:6-16):
// H2D of the row inputs, one cooperative launch in decoder-step mode, D2H of
// the logits [4][V] and the next positions.  The caches are the engine's
// resident K/V, or device buffers of the caller in the same layout.
int32_t run_decoder_step(Engine *e, const int64_t *token, const int64_t *position, const int32_t *seq_len,
                         void *key_cache, const int32_t *slot, const int32_t *active, const int32_t *block_table,
                         void *value_cache, float *logits_out, int64_t *next_position_out) {
  const ModelDims &m = e->m;
  cudaSetDevice(e->device);
  if (e->tp_size > 1) {
    e->last_error = "cruise_decoder_step: single-GPU engines only (no tensor parallelism)";
    return -4;
  }
  auto reject = [&](const std::string &why) {
    e->last_error = "cruise_decoder_step: " + why;
    return -1;
  };
  for (int i = 0; i < kBatch * m.bpr; ++i)
    if (block_table[i] < 0 || block_table[i] >= m.NB) return reject("block table entry outside the cache");
  for (int b = 0; b < kBatch; ++b) {
    // every row's embedding row is gathered, so every token must exist
    if (token[b] < 0 || token[b] >= m.V) return reject("token id outside the vocabulary");
    if (active[b] != 0 && active[b] != 1) return reject("active flags must be 0 or 1");
    if (seq_len[b] < 0 || seq_len[b] > m.C) return reject("sequence length outside [0, capacity]");
    if (active[b] == 0) continue;
    if (position[b] < 0 || position[b] >= m.C) return reject("position of an active row outside [0, capacity)");
    // the new K/V are written at slot[row] and read back at the row's position:
    // the two must be the same cache slot (what the reference's callers pass)
    const int64_t logical = position[b] / m.bs;
    const int64_t expect = static_cast<int64_t>(block_table[b * m.bpr + logical]) * m.bs + position[b] % m.bs;
    if (slot[b] != expect) return reject("slot of an active row is not its position's block-table slot");
  }
  for (void *cache : {key_cache, value_cache}) {
    if (cache == nullptr) continue;
    cudaPointerAttributes attr{};
    if (cudaPointerGetAttributes(&attr, cache) != cudaSuccess || attr.type != cudaMemoryTypeDevice ||
        attr.device != e->device || (reinterpret_cast<uintptr_t>(cache) & 15) != 0) {
      cudaGetLastError();
      return reject("caches must be 16-byte aligned device memory on the engine's device");
    }
  }
  if ((key_cache == nullptr) != (value_cache == nullptr)) return reject("pass both caches or neither");
  EpochIO *io = e->h_io;
  std::memset(io, 0, sizeof(EpochIO));
  std::memcpy(io->token, token, sizeof(io->token));
  std::memcpy(io->position, position, sizeof(io->position));
  std::memcpy(io->seq_len, seq_len, sizeof(io->seq_len));
  std::memcpy(io->slot, slot, sizeof(io->slot));
  std::memcpy(io->active, active, sizeof(io->active));
  std::memcpy(io->block_table, block_table, sizeof(int32_t) * kBatch * m.bpr);
  cudaError_t err = cudaMemcpyAsync(e->d_io, io, offsetof(EpochIO, history), cudaMemcpyHostToDevice, e->stream);
  if (err == cudaSuccess) err = cudaMemsetAsync(e->d_sync, 0, sync_bytes(e->sms), e->stream);
  if (err != cudaSuccess) return set_err(e, err, "decoder step inputs");
  EpochParams p = engine_params(e);
  p.mode = kModeDecoderStep;
  p.trace = nullptr;
  p.trace_cta = nullptr;
  p.logits = e->logits;
  if (key_cache != nullptr) {
    p.key_cache = static_cast<bf16 *>(key_cache);
    p.value_cache = static_cast<bf16 *>(value_cache);
  }
  p.timeout_ns = 2000000000ull;
  p.tp_size = 1;
  p.launch_id = ++e->launches;
  void *args[] = {&p};
  cudaEventRecord(e->ev0, e->stream);
  err = cudaLaunchCooperativeKernel(reinterpret_cast<const void *>(resident_epoch_kernel), dim3(e->sms),
                                    dim3(kThreads), args, e->smem, e->stream);
  cudaEventRecord(e->ev1, e->stream);
  if (err != cudaSuccess) return set_err(e, err, "decoder step launch");
  err = cudaMemcpyAsync(&io->history, &e->d_io->history, sizeof(EpochIO) - offsetof(EpochIO, history),
                        cudaMemcpyDeviceToHost, e->stream);
  if (err == cudaSuccess)
    err = cudaMemcpyAsync(logits_out, e->logits, sizeof(float) * kBatch * m.V, cudaMemcpyDeviceToHost, e->stream);
  if (err == cudaSuccess) err = cudaStreamSynchronize(e->stream);
  if (err != cudaSuccess) return set_err(e, err, "decoder step completion");
  cudaEventElapsedTime(&e->last_ms, e->ev0, e->ev1);
  e->last_launches = 1;
  if (io->control_out[3] != kOk) {
    e->last_error = "cruise_decoder_step: a device-side wait gave up (status " + std::to_string(io->control_out[3]) + ")";
    return -3;
  }
  std::memcpy(next_position_out, io->history, sizeof(int64_t) * kBatch);
  return 0;
}

// ---- reference bridge helpers (native/resident_epoch_bridge.cpp) -----------------------------
#pragma pack(push, 1)
struct TransferHeader {   // :73-89
  uint64_t magic;
  uint32_t version;
  uint32_t header_bytes;
  uint64_t transfer_id;
  uint64_t payload_bytes;
  uint32_t import_mask;
  int32_t row_generations[kBatch];
  uint32_t layers, batch_size, block_size, kv_heads, head_size, element_bytes;
  uint32_t checksum;
};
#pragma pack(pop)
static_assert(sizeof(TransferHeader) == CRUISE_RESIDENT_TRANSFER_HEADER_BYTES, "transfer header ABI");
static_assert(offsetof(EpochIO, history) == 616, "epoch input block: 616 bytes host-to-device per epoch");
static_assert(sizeof(EpochIO) - offsetof(EpochIO, history) == 368, "epoch output block: 368 bytes per epoch");
static_assert(sizeof(ResidentEpochIpcMetadata) == CRUISE_RESIDENT_IPC_METADATA_BYTES, "IPC metadata ABI");

std::mutex g_lifecycle_mutex;
bool g_bridge_active = false;

struct BridgeEngine {
  Engine *engine = nullptr;
  std::map<std::string, void *> ipc_imports;
  int32_t prefill_mask = 0;   // rows resident_epoch_prefill left in the device staging for the next execute
  int32_t prefill_lens[kBatch] = {};   // their prompt lengths: the import epoch decodes from len - 1
};

bool read_transfer(const Engine *e, const char *path, uint64_t transfer_id, const int32_t *gens,
                   std::vector<uint8_t> &payload, int32_t &mask, uint32_t &checksum) {   // :108-154
  if (path == nullptr || gens == nullptr || transfer_id == 0 || std::strncmp(path, "/dev/shm/", 9) != 0)
    return false;
  const uint64_t payload_bytes = static_cast<uint64_t>(import_payload_bytes(e));
  std::ifstream stream(path, std::ios::binary | std::ios::ate);
  if (!stream || static_cast<uint64_t>(stream.tellg()) != CRUISE_RESIDENT_TRANSFER_HEADER_BYTES + payload_bytes)
    return false;
  stream.seekg(0, std::ios::beg);
  TransferHeader h{};
  stream.read(reinterpret_cast<char *>(&h), sizeof(h));
  if (!stream || h.magic != CRUISE_RESIDENT_TRANSFER_MAGIC || h.version != CRUISE_RESIDENT_TRANSFER_VERSION ||
      h.header_bytes != CRUISE_RESIDENT_TRANSFER_HEADER_BYTES || h.transfer_id != transfer_id ||
      h.payload_bytes != payload_bytes || h.import_mask == 0 || h.import_mask >= (1u << kBatch) ||
      h.layers != static_cast<uint32_t>(e->m.L) || h.batch_size != kBatch ||
      h.block_size != static_cast<uint32_t>(e->m.bs) || h.kv_heads != static_cast<uint32_t>(e->m.nkv) ||
      h.head_size != static_cast<uint32_t>(e->m.d) || h.element_bytes != 2 || h.checksum == 0)
    return false;
  for (int r = 0; r < kBatch; ++r) {
    const bool sel = (h.import_mask & (1u << r)) != 0;
    if (sel) {
      if (h.row_generations[r] <= 0 || h.row_generations[r] != gens[r]) return false;
    } else if (h.row_generations[r] != 0) {
      return false;
    }
  }
  payload.resize(payload_bytes);
  stream.read(reinterpret_cast<char *>(payload.data()), static_cast<std::streamsize>(payload.size()));
  if (!stream) return false;
  mask = static_cast<int32_t>(h.import_mask);
  checksum = h.checksum;
  return true;
}

bool validate_ipc(const Engine *e, const ResidentEpochIpcMetadata *md, const int32_t *gens) {   // :156-199
  if (md == nullptr || gens == nullptr || md->magic != CRUISE_RESIDENT_IPC_METADATA_MAGIC ||
      md->version != CRUISE_RESIDENT_IPC_METADATA_VERSION || md->source_bytes == 0 || md->import_mask == 0 ||
      md->import_mask >= (1u << kBatch))
    return false;
  if (e->m.L * 2 > CRUISE_RESIDENT_IPC_KEY_COUNT) return false;
  const uint64_t block_bytes = static_cast<uint64_t>(e->m.bs) * e->m.nkv * e->m.d * 2;
  for (int r = 0; r < kBatch; ++r) {
    const bool sel = (md->import_mask & (1u << r)) != 0;
    if (sel) {
      if (md->row_generations[r] <= 0 || md->row_generations[r] != gens[r] || md->block_ids[r] < 0) return false;
    } else if (md->row_generations[r] != 0 || md->block_ids[r] != 0) {
      return false;
    }
  }
  for (int i = 0; i < 2 * e->m.L; ++i) {
    for (int r = 0; r < kBatch; ++r) {
      if ((md->import_mask & (1u << r)) == 0) continue;
      const uint64_t end = (static_cast<uint64_t>(md->block_ids[r]) + 1u) * block_bytes;
      if (md->source_offsets[i] > md->source_bytes || end > md->source_bytes - md->source_offsets[i]) return false;
    }
  }
  return true;
}

// Opens the exporting process's K/V allocations (cudaIpcMemHandle_t in each
// 64-byte key) and gathers the selected blocks into the import staging buffer
// with device-to-device copies (:218-273).
bool prepare_ipc_payload(BridgeEngine *be, const ResidentEpochIpcMetadata *md) {
  Engine *e = be->engine;
  const size_t bytes = static_cast<size_t>(import_payload_bytes(e));
  if (e->d_payload == nullptr) {
    if (cudaMalloc(&e->d_payload, bytes) != cudaSuccess) return false;
    e->payload_bytes = bytes;
  }
  if (cudaMemsetAsync(e->d_payload, 0, bytes, e->stream) != cudaSuccess) return false;
  const size_t block_bytes = static_cast<size_t>(e->m.bs) * e->m.nkv * e->m.d * 2;
  const size_t cache_bytes = bytes / 2;
  for (int layer = 0; layer < e->m.L; ++layer) {
    void *src[2] = {nullptr, nullptr};
    for (int kvi = 0; kvi < 2; ++kvi) {
      const std::string key(md->keys[layer * 2 + kvi], CRUISE_RESIDENT_IPC_KEY_BYTES);
      auto it = be->ipc_imports.find(key);
      if (it == be->ipc_imports.end()) {
        cudaIpcMemHandle_t handle;
        std::memcpy(&handle, md->keys[layer * 2 + kvi], sizeof(handle));
        void *ptr = nullptr;
        if (cudaIpcOpenMemHandle(&ptr, handle, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return false;
        it = be->ipc_imports.emplace(key, ptr).first;
      }
      src[kvi] = it->second;
    }
    for (int r = 0; r < kBatch; ++r) {
      if ((md->import_mask & (1u << r)) == 0) continue;
      const size_t off = static_cast<size_t>(md->block_ids[r]) * block_bytes;
      const size_t row_off = (static_cast<size_t>(layer) * kBatch + r) * block_bytes;
      for (int kvi = 0; kvi < 2; ++kvi) {
        const uint8_t *s = static_cast<const uint8_t *>(src[kvi]) + md->source_offsets[layer * 2 + kvi] + off;
        if (cudaMemcpyAsync(e->d_payload + kvi * cache_bytes + row_off, s, block_bytes, cudaMemcpyDeviceToDevice,
                            e->stream) != cudaSuccess)
          return false;
      }
    }
  }
  return true;
}

int64_t process_cpu_us() {
  timespec v{};
  if (clock_gettime(CLOCK_PROCESS_CPUTIME_ID, &v) != 0) return -1;
  return static_cast<int64_t>(v.tv_sec) * 1000000LL + v.tv_nsec / 1000;
}

int32_t preset(const char *name, CruiseModelConfig *cfg) {
  if (name == nullptr || cfg == nullptr) return -1;
  std::memset(cfg, 0, sizeof(*cfg));
  cfg->rms_eps = 1e-6f;
  cfg->rope_theta = 1000000.0f;
  cfg->blocks_per_row = 2;
  cfg->num_blocks = 8;
  if (std::strcmp(name, "qwen2.5-7b") == 0) {
    cfg->num_layers = 28; cfg->hidden = 3584; cfg->num_heads = 28; cfg->num_kv_heads = 4;
    cfg->head_dim = 128; cfg->intermediate = 18944; cfg->vocab = 152064; cfg->block_size = 128;
    cfg->configured_eos = 151645;
    return 0;
  }
  if (std::strcmp(name, "tiny") == 0) {
    cfg->num_layers = 2; cfg->hidden = 256; cfg->num_heads = 4; cfg->num_kv_heads = 2;
    cfg->head_dim = 64; cfg->intermediate = 688; cfg->vocab = 4096; cfg->block_size = 16;
    cfg->configured_eos = 4095;
    return 0;
  }
  return -1;
}

}  // namespace
}  // namespace cruise

// ===================================== allocation-free epoch ======================================
// Scratch of cruise_epoch_run_noalloc, sized once at build time.  Each GPU on
// which this library's device code is loaded holds these bytes until the
// process exits.  Host code names the array only to look up its device address.
constexpr size_t kNoAllocScratchBytes = size_t(1) << 20;
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

namespace cruise {
namespace {

constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mutex;
void *g_noalloc_base[kNoAllocMaxDevices] = {};

// Device address of the static scratch on `device`, which must be current.  The
// lookup runs once per device, on that device's first allocation-free call, and
// the address is kept for the life of the process: after a cudaDeviceReset
// (which creates a new primary context) the allocation-free call must not be
// used again in this process.
cudaError_t noalloc_base(int device, void **base) {
  if (device < 0 || device >= kNoAllocMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (g_noalloc_base[device] == nullptr) {
    void *ptr = nullptr;
    const cudaError_t err = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (err != cudaSuccess) return err;
    g_noalloc_base[device] = ptr;
  }
  *base = g_noalloc_base[device];
  return cudaSuccess;
}

// Offsets in the static scratch of everything one epoch uses besides the
// engine's model state (weights, KV cache, RoPE tables, resident row state).
struct NoAllocLayout {
  size_t io, work, sync, h, qkv, attn, act, av, ai, ab, total;
};

NoAllocLayout noalloc_layout(const Engine *e) {
  const ModelDims &m = e->m;
  NoAllocLayout l{};
  size_t st = 0;
  auto take = [&](size_t bytes) {
    const size_t off = st;
    st = align_up(st + bytes, 256);
    return off;
  };
  l.io = take(sizeof(EpochIO));
  l.work = take(sizeof(EpochWork));
  l.sync = take(sync_bytes(e->sms));   // SyncState, then the tagged partial-sum words
  l.h = take(static_cast<size_t>(kBatch) * m.H * 2);
  l.qkv = take(static_cast<size_t>(kBatch) * m.Nqkv * 2);
  l.attn = take(static_cast<size_t>(kBatch) * m.H * 2);
  l.act = take(static_cast<size_t>(kBatch) * m.I_pad * 2);
  l.av = take(static_cast<size_t>(e->sms) * kBatch * 4);
  l.ai = take(static_cast<size_t>(e->sms) * kBatch * 4);
  l.ab = take(static_cast<size_t>(e->sms) * kBatch * 4);
  l.total = st;
  return l;
}

}  // namespace

// One greedy epoch whose scratch is the static array instead of the engine's
// allocation; inputs and outputs are host arrays as in run_epoch.
int32_t run_epoch_noalloc(Engine *e, const int64_t *token, const int64_t *position, const int32_t *seq_len,
                          const int32_t *slot, const int32_t *active, const int32_t *block_table,
                          const int32_t *control, int64_t *history, int32_t *control_out) {
  cudaError_t err = cudaSetDevice(e->device);
  if (err != cudaSuccess) return set_err(e, err, "noalloc set device");
  if (e->tp_size > 1) {
    e->last_error = "cruise_epoch_run_noalloc: single-GPU engines only (no tensor parallelism)";
    return -4;
  }
  const NoAllocLayout l = noalloc_layout(e);
  if (l.total > kNoAllocScratchBytes) {
    e->last_error = "cruise_epoch_run_noalloc: this model needs " + std::to_string(l.total) +
                    " bytes of scratch, the static scratch holds " + std::to_string(kNoAllocScratchBytes);
    return -2;
  }
  if ((control[2 + kBatch] & kImportFlag) != 0) {
    e->last_error = "cruise_epoch_run_noalloc: a KV import needs the payload staging of cruise_epoch_run";
    return -3;
  }
  void *base = nullptr;
  err = noalloc_base(e->device, &base);
  if (err != cudaSuccess) return set_err(e, err, "noalloc scratch address");
  uint8_t *sb = static_cast<uint8_t *>(base);
  EpochIO io;
  std::memset(&io, 0, sizeof(io));
  std::memcpy(io.token, token, sizeof(io.token));
  std::memcpy(io.position, position, sizeof(io.position));
  std::memcpy(io.seq_len, seq_len, sizeof(io.seq_len));
  std::memcpy(io.slot, slot, sizeof(io.slot));
  std::memcpy(io.active, active, sizeof(io.active));
  std::memcpy(io.block_table, block_table, sizeof(int32_t) * kBatch * e->m.bpr);
  std::memcpy(io.control, control, sizeof(io.control));
  // every call starts from zeroed scratch: grid-barrier counters, split-partial
  // flags, error word and the padded activation columns must read zero
  err = cudaMemsetAsync(sb, 0, l.total, e->stream);
  if (err == cudaSuccess)
    err = cudaMemcpyAsync(sb + l.io, &io, offsetof(EpochIO, history), cudaMemcpyHostToDevice, e->stream);
  if (err != cudaSuccess) return set_err(e, err, "noalloc epoch inputs");

  EpochParams p{};
  p.m = e->m;
  p.layers = e->d_layers;
  p.embed = e->embed;
  p.final_norm = e->final_norm;
  p.lm_head = e->lm_head;
  p.rope_cos = e->rope_cos;
  p.rope_sin = e->rope_sin;
  p.key_cache = e->key_cache;
  p.value_cache = e->value_cache;
  p.h = reinterpret_cast<bf16 *>(sb + l.h);
  p.qkv = reinterpret_cast<bf16 *>(sb + l.qkv);
  p.attn = reinterpret_cast<bf16 *>(sb + l.attn);
  p.act = reinterpret_cast<bf16 *>(sb + l.act);
  p.partials = reinterpret_cast<uint64_t *>(sb + l.sync + sizeof(SyncState));
  p.arg_val = reinterpret_cast<float *>(sb + l.av);
  p.arg_idx = reinterpret_cast<int32_t *>(sb + l.ai);
  p.arg_bad = reinterpret_cast<int32_t *>(sb + l.ab);
  p.logits = nullptr;
  p.import_payload = nullptr;
  p.io = reinterpret_cast<EpochIO *>(sb + l.io);
  p.res = e->d_res;
  p.work = reinterpret_cast<EpochWork *>(sb + l.work);
  p.sync = reinterpret_cast<SyncState *>(sb + l.sync);
  p.grid = e->sms;
  p.stages = e->stages;
  p.xs_stride = e->xs_stride;
  p.down_xglobal = e->down_xglobal;
  p.o_xglobal = e->o_xglobal;
  p.trace = nullptr;
  p.timeout_ns = 2000000000ull;   // every device-side wait gives up after 2 s
  p.l2_ahead = e->l2_ahead;
  p.l2_hints = e->l2_hints;
  p.tp_size = 1;
  void *args[] = {&p};
  cudaEventRecord(e->ev0, e->stream);
  err = cudaLaunchCooperativeKernel(reinterpret_cast<const void *>(resident_epoch_kernel), dim3(e->sms),
                                    dim3(kThreads), args, e->smem, e->stream);
  cudaEventRecord(e->ev1, e->stream);
  if (err != cudaSuccess) return set_err(e, err, "noalloc epoch launch");
  err = cudaMemcpyAsync(&io.history, sb + l.io + offsetof(EpochIO, history),
                        sizeof(EpochIO) - offsetof(EpochIO, history), cudaMemcpyDeviceToHost, e->stream);
  // the error word and the site of the wait that gave up, for a 207 status
  uint32_t words[2] = {0, 0};
  if (err == cudaSuccess)
    err = cudaMemcpyAsync(words, sb + l.sync + offsetof(SyncState, error), sizeof(words), cudaMemcpyDeviceToHost,
                          e->stream);
  if (err == cudaSuccess) err = cudaStreamSynchronize(e->stream);
  if (err != cudaSuccess) return set_err(e, err, "noalloc epoch completion");
  cudaEventElapsedTime(&e->last_ms, e->ev0, e->ev1);
  e->last_launches = 1;
  std::memcpy(history, io.history, sizeof(io.history));
  std::memcpy(control_out, io.control_out, sizeof(io.control_out));
  if (control_out[3] == kModelError && words[0])
    e->last_error = "epoch ended by a device-side wait that gave up (site " + std::to_string(words[1]) + ")";
  return 0;
}

}  // namespace cruise

using cruise::BridgeEngine;
using cruise::Engine;
using cruise::kBatch;
using cruise::kMaxSteps;

// ===================================== C ABI =========================================================
extern "C" {

int32_t cruise_epoch_preset(const char *name, CruiseModelConfig *cfg) { return cruise::preset(name, cfg); }

void *cruise_epoch_create_tp(const CruiseModelConfig *cfg, int32_t device, int32_t tp_rank, int32_t tp_size,
                             int32_t *status) {
  int32_t dummy = 0;
  if (status == nullptr) status = &dummy;
  *status = 1;
  if (cfg == nullptr) return nullptr;
  return cruise::create_engine(*cfg, device, status, tp_rank, tp_size);
}

int32_t cruise_epoch_tp_handle(void *engine, void *handle_out) {
  if (engine == nullptr || handle_out == nullptr) return -1;
  Engine *e = static_cast<Engine *>(engine);
  if (e->tp_size < 2) return -1;
  cudaSetDevice(e->device);
  cudaIpcMemHandle_t handle;
  const cudaError_t err = cudaIpcGetMemHandle(&handle, e->xchg);
  if (err != cudaSuccess) return cruise::set_err(e, err, "tp handle");
  std::memcpy(handle_out, &handle, sizeof(handle));
  return 0;
}

int32_t cruise_epoch_tp_connect(void *engine, const void *handles) {
  if (engine == nullptr || handles == nullptr) return -1;
  Engine *e = static_cast<Engine *>(engine);
  if (e->tp_size < 2 || e->tp_connected) return -1;
  std::lock_guard<std::mutex> lock(e->execute_mutex);
  cudaSetDevice(e->device);
  std::vector<cruise::TpExchange *> peers(cruise::kMaxTp, nullptr);
  for (int r = 0; r < e->tp_size; ++r) {
    if (r == e->tp_rank) {
      peers[r] = e->xchg;
      continue;
    }
    cudaIpcMemHandle_t handle;
    std::memcpy(&handle, static_cast<const uint8_t *>(handles) + static_cast<size_t>(r) * sizeof(handle),
                sizeof(handle));
    void *ptr = nullptr;
    const cudaError_t err = cudaIpcOpenMemHandle(&ptr, handle, cudaIpcMemLazyEnablePeerAccess);
    if (err != cudaSuccess) return cruise::set_err(e, err, "tp connect: open peer exchange block");
    e->opened.push_back(ptr);
    peers[r] = static_cast<cruise::TpExchange *>(ptr);
  }
  const cudaError_t err = cruise::copy_sync(e, e->d_peers, peers.data(), sizeof(cruise::TpExchange *) * cruise::kMaxTp,
                                            cudaMemcpyHostToDevice);
  if (err != cudaSuccess) return cruise::set_err(e, err, "tp connect");
  e->tp_connected = true;
  return 0;
}

int32_t cruise_epoch_tp_shard(const CruiseModelConfig *cfg, int32_t tp_rank, int32_t tp_size, int32_t *shard_out) {
  if (cfg == nullptr || shard_out == nullptr) return -1;
  cruise::TpGeom g{};
  if (!cruise::tp_geometry(*cfg, tp_rank, tp_size, g)) return -1;
  const int32_t v[8] = {g.q0, g.nq, g.kv0, g.nkv, g.i0, g.ni, g.v0, g.nv};
  std::memcpy(shard_out, v, sizeof(v));
  return 0;
}

void *cruise_epoch_create(const CruiseModelConfig *cfg, int32_t device, int32_t *status) {
  int32_t dummy = 0;
  if (status == nullptr) status = &dummy;
  *status = 1;
  if (cfg == nullptr) return nullptr;
  return cruise::create_engine(*cfg, device, status);
}

void cruise_epoch_destroy(void *engine) { cruise::destroy_engine(static_cast<Engine *>(engine)); }

int32_t cruise_epoch_init_synthetic(void *engine, uint64_t seed, double stddev) {
  if (engine == nullptr) return -1;
  Engine *e = static_cast<Engine *>(engine);
  std::lock_guard<std::mutex> lock(e->execute_mutex);
  cudaSetDevice(e->device);
  return cruise::synth_all(e, seed, stddev);
}

int32_t cruise_epoch_set_weight(void *engine, const char *name, const void *host_bf16, uint64_t bytes) {
  if (engine == nullptr || name == nullptr || host_bf16 == nullptr) return -1;
  Engine *e = static_cast<Engine *>(engine);
  std::lock_guard<std::mutex> lock(e->execute_mutex);
  cudaSetDevice(e->device);
  return cruise::copy_tensor(e, name, const_cast<void *>(host_bf16), bytes, true);
}

int32_t cruise_epoch_get_weight(void *engine, const char *name, void *host_bf16, uint64_t bytes) {
  if (engine == nullptr || name == nullptr || host_bf16 == nullptr) return -1;
  Engine *e = static_cast<Engine *>(engine);
  std::lock_guard<std::mutex> lock(e->execute_mutex);
  cudaSetDevice(e->device);
  return cruise::copy_tensor(e, name, host_bf16, bytes, false);
}

int32_t cruise_epoch_set_rope_table(void *engine, const uint16_t *cos_bf16, const uint16_t *sin_bf16,
                                    uint64_t bytes) {
  if (engine == nullptr || cos_bf16 == nullptr || sin_bf16 == nullptr) return -1;
  Engine *e = static_cast<Engine *>(engine);
  if (bytes != static_cast<uint64_t>(e->m.C) * e->m.d * 2) return -1;
  std::lock_guard<std::mutex> lock(e->execute_mutex);
  cudaSetDevice(e->device);
  cudaError_t err = cruise::copy_sync(e, e->rope_cos, cos_bf16, bytes, cudaMemcpyHostToDevice);
  if (err == cudaSuccess) err = cruise::copy_sync(e, e->rope_sin, sin_bf16, bytes, cudaMemcpyHostToDevice);
  return cruise::set_err(e, err, "rope table");
}

int32_t cruise_epoch_read_kv(void *engine, void *key_host, void *value_host, uint64_t bytes_each) {
  if (engine == nullptr || key_host == nullptr || value_host == nullptr) return -1;
  Engine *e = static_cast<Engine *>(engine);
  const uint64_t expect = static_cast<uint64_t>(e->m.L) * e->m.NB * e->m.bs * e->m.nkv * e->m.d * 2;
  if (bytes_each != expect) return -1;
  std::lock_guard<std::mutex> lock(e->execute_mutex);
  cudaSetDevice(e->device);
  cudaError_t err = cruise::copy_sync(e, key_host, e->key_cache, bytes_each, cudaMemcpyDeviceToHost);
  if (err == cudaSuccess) err = cruise::copy_sync(e, value_host, e->value_cache, bytes_each, cudaMemcpyDeviceToHost);
  return cruise::set_err(e, err, "read kv");
}

int32_t cruise_epoch_write_kv(void *engine, const void *key_host, const void *value_host, uint64_t bytes_each) {
  if (engine == nullptr || key_host == nullptr || value_host == nullptr) return -1;
  Engine *e = static_cast<Engine *>(engine);
  const uint64_t expect = static_cast<uint64_t>(e->m.L) * e->m.NB * e->m.bs * e->m.nkv * e->m.d * 2;
  if (bytes_each != expect) return -1;
  std::lock_guard<std::mutex> lock(e->execute_mutex);
  cudaSetDevice(e->device);
  cudaError_t err = cruise::copy_sync(e, e->key_cache, key_host, bytes_each, cudaMemcpyHostToDevice);
  if (err == cudaSuccess) err = cruise::copy_sync(e, e->value_cache, value_host, bytes_each, cudaMemcpyHostToDevice);
  return cruise::set_err(e, err, "write kv");
}

int32_t cruise_epoch_run(void *engine, const int64_t *token, const int64_t *position, const int32_t *seq_len,
                         const int32_t *slot, const int32_t *active, const int32_t *block_table,
                         const uint8_t *tiling, const int32_t *control, const void *import_payload,
                         uint64_t import_bytes, const int64_t *forced_tokens, int64_t *history,
                         int32_t *control_out, float *logits_out) {
  if (engine == nullptr || token == nullptr || position == nullptr || seq_len == nullptr || slot == nullptr ||
      active == nullptr || block_table == nullptr || control == nullptr || history == nullptr ||
      control_out == nullptr)
    return -1;
  Engine *e = static_cast<Engine *>(engine);
  std::lock_guard<std::mutex> lock(e->execute_mutex);
  return cruise::run_epoch(e, token, position, seq_len, slot, active, block_table, tiling, control,
                           import_payload, import_bytes, history, control_out, logits_out, forced_tokens);
}

int32_t cruise_epoch_run_noalloc(void *engine, const int64_t *token, const int64_t *position,
                                 const int32_t *seq_len, const int32_t *slot, const int32_t *active,
                                 const int32_t *block_table, const int32_t *control, int64_t *history,
                                 int32_t *control_out) {
  if (engine == nullptr || token == nullptr || position == nullptr || seq_len == nullptr || slot == nullptr ||
      active == nullptr || block_table == nullptr || control == nullptr || history == nullptr ||
      control_out == nullptr)
    return -1;
  Engine *e = static_cast<Engine *>(engine);
  std::lock_guard<std::mutex> lock(e->execute_mutex);
  return cruise::run_epoch_noalloc(e, token, position, seq_len, slot, active, block_table, control, history,
                                   control_out);
}

int32_t cruise_decoder_step(void *engine, const int64_t *token, const int64_t *position, const int32_t *seq_len,
                            void *key_cache, const int32_t *slot, const int32_t *active,
                            const int32_t *block_table, void *value_cache, const uint8_t *tiling,
                            float *logits_out, int64_t *next_position_out) {
  (void)tiling;   // the ABI's 72-byte tiling blob: accepted, not needed
  if (engine == nullptr || token == nullptr || position == nullptr || seq_len == nullptr || slot == nullptr ||
      active == nullptr || block_table == nullptr || logits_out == nullptr || next_position_out == nullptr)
    return -1;
  Engine *e = static_cast<Engine *>(engine);
  std::lock_guard<std::mutex> lock(e->execute_mutex);
  return cruise::run_decoder_step(e, token, position, seq_len, key_cache, slot, active, block_table, value_cache,
                                  logits_out, next_position_out);
}

int32_t cruise_epoch_last_timing(void *engine, double *device_us, int32_t *kernel_launches) {
  if (engine == nullptr) return -1;
  Engine *e = static_cast<Engine *>(engine);
  if (device_us) *device_us = static_cast<double>(e->last_ms) * 1000.0;
  if (kernel_launches) *kernel_launches = e->last_launches;
  return 0;
}

int32_t cruise_epoch_set_trace(void *engine, int32_t enable) {
  if (engine == nullptr) return -1;
  Engine *e = static_cast<Engine *>(engine);
  std::lock_guard<std::mutex> lock(e->execute_mutex);
  if (enable == 2 && e->trace_cta == nullptr) {
    cudaSetDevice(e->device);
    const cudaError_t err = cudaMalloc(&e->trace_cta, static_cast<size_t>(cruise::kTraceMax) * e->sms * cruise::kTraceCtaWords * sizeof(uint32_t));
    if (err != cudaSuccess) {
      e->trace_cta = nullptr;
      return cruise::set_err(e, err, "per-CTA trace buffer");
    }
  }
  e->trace_on = enable != 0;
  e->trace_cta_on = enable == 2;
  return 0;
}

int32_t cruise_epoch_read_trace_cta(void *engine, uint32_t *stamps, int32_t barriers, int32_t *ctas) {
  if (engine == nullptr || ctas == nullptr || barriers < 0 || barriers > cruise::kTraceMax ||
      (stamps == nullptr && barriers > 0))
    return -1;
  Engine *e = static_cast<Engine *>(engine);
  std::lock_guard<std::mutex> lock(e->execute_mutex);
  *ctas = e->sms;
  if (barriers == 0) return 0;
  if (e->trace_cta == nullptr) return -1;
  cudaSetDevice(e->device);
  const cudaError_t err = cruise::copy_sync(e, stamps, e->trace_cta,
                                            static_cast<size_t>(barriers) * e->sms * cruise::kTraceCtaWords * sizeof(uint32_t),
                                            cudaMemcpyDeviceToHost);
  return cruise::set_err(e, err, "read per-CTA trace");
}

int32_t cruise_epoch_prefill(void *engine, const int64_t *prompt_tokens, const int32_t *prompt_lens,
                             int32_t stride) {
  if (engine == nullptr || prompt_lens == nullptr || (prompt_tokens == nullptr && stride != 0) || stride < 0)
    return -1;
  Engine *e = static_cast<Engine *>(engine);
  std::lock_guard<std::mutex> lock(e->execute_mutex);
  cudaSetDevice(e->device);
  return cruise::prefill_run(e, prompt_tokens, prompt_lens, stride);
}

int32_t cruise_epoch_stream_enable(void *engine, int32_t enable) {
  if (engine == nullptr) return -1;
  Engine *e = static_cast<Engine *>(engine);
  std::lock_guard<std::mutex> lock(e->execute_mutex);
  if (enable != 0 && e->h_stream == nullptr) {
    cudaSetDevice(e->device);
    void *host = nullptr, *dev = nullptr;
    cudaError_t err = cudaHostAlloc(&host, sizeof(cruise::StreamRing), cudaHostAllocMapped);
    if (err == cudaSuccess) err = cudaHostGetDevicePointer(&dev, host, 0);
    if (err != cudaSuccess) {
      if (host != nullptr) cudaFreeHost(host);
      return cruise::set_err(e, err, "stream ring");
    }
    std::memset(host, 0, sizeof(cruise::StreamRing));
    e->h_stream = static_cast<cruise::StreamRing *>(host);
    e->d_stream = static_cast<cruise::StreamRing *>(dev);
  }
  e->stream_on = enable != 0;
  return 0;
}

uint32_t cruise_epoch_stream_next_id(void *engine) {
  if (engine == nullptr) return 0;
  return static_cast<Engine *>(engine)->launches.load() + 1;
}

int32_t cruise_epoch_stream_poll(void *engine, uint32_t launch_id, int64_t *tokens_out) {
  if (engine == nullptr || tokens_out == nullptr) return -1;
  const Engine *e = static_cast<const Engine *>(engine);
  if (e->h_stream == nullptr) return -1;
  // no lock: the epoch that publishes holds the engine's mutex while it runs
  const uint64_t published = *reinterpret_cast<const volatile uint64_t *>(&e->h_stream->published);
  std::atomic_thread_fence(std::memory_order_acquire);
  if (static_cast<uint32_t>(published >> 32) != launch_id) return 0;
  const int32_t steps = std::min(static_cast<int32_t>(published & 0xFFFFFFFFu), cruise::kMaxSteps);
  for (int i = 0; i < steps * cruise::kBatch; ++i)
    tokens_out[i] = reinterpret_cast<const volatile int64_t *>(&e->h_stream->tokens[0][0])[i];
  return steps;
}

int32_t cruise_epoch_read_trace(void *engine, int32_t series, uint64_t *ns, int32_t count) {
  if (engine == nullptr || ns == nullptr || series < 0 || series >= cruise::kTraceSeries || count < 0 || count > cruise::kTraceMax)
    return -1;
  Engine *e = static_cast<Engine *>(engine);
  std::lock_guard<std::mutex> lock(e->execute_mutex);
  cudaSetDevice(e->device);
  cudaError_t err = cruise::copy_sync(e, ns, e->trace + static_cast<size_t>(series) * cruise::kTraceMax,
                                      sizeof(uint64_t) * count, cudaMemcpyDeviceToHost);
  return cruise::set_err(e, err, "read trace");
}

const char *cruise_epoch_last_error(void *engine) {
  if (engine == nullptr) return cruise::g_create_error.c_str();
  return static_cast<Engine *>(engine)->last_error.c_str();
}

// ---- reference-compatible bridge ----------------------------------------------------------------------
void *resident_epoch_create(const char *air_path, const char *graph_config, const char *func_config,
                            const char *external_weight_dir, const char *tiling_path, int32_t *status) {
  (void)graph_config;
  (void)func_config;
  if (status == nullptr) return nullptr;
  *status = 1;
  std::lock_guard<std::mutex> lifecycle(cruise::g_lifecycle_mutex);
  cruise::g_create_error.clear();
  if (cruise::g_bridge_active || air_path == nullptr || external_weight_dir == nullptr) {
    cruise::g_create_error = cruise::g_bridge_active ? "a resident epoch is already active in this process"
                                                     : "null model or weight path";
    return nullptr;
  }
  CruiseModelConfig cfg{};
  if (cruise::preset(air_path, &cfg) != 0) {
    *status = 5;
    cruise::g_create_error = std::string("unknown model preset ") + air_path;
    return nullptr;
  }
  std::array<uint8_t, cruise::kTilingBytes> tiling{};
  if (tiling_path != nullptr && tiling_path[0] != '\0') {
    std::ifstream t(tiling_path, std::ios::binary | std::ios::ate);
    t.seekg(0, std::ios::beg);
    if (t) t.read(reinterpret_cast<char *>(tiling.data()), tiling.size());
    if (!t || t.gcount() != static_cast<std::streamsize>(tiling.size()) || t.peek() != EOF) {
      *status = 2;
      cruise::g_create_error = "tiling file missing or not " + std::to_string(tiling.size()) + " bytes";
      return nullptr;
    }
  }
  Engine *e = cruise::create_engine(cfg, 0, status);
  if (e == nullptr) return nullptr;
  e->tiling = tiling;
  const std::string weights(external_weight_dir);
  int32_t rc = 0;
  if (weights.rfind("synthetic:", 0) == 0) {
    rc = cruise::synth_all(e, std::strtoull(weights.c_str() + 10, nullptr, 10), 0.02);
  } else {
    // one raw bf16 file per checkpoint tensor
    std::vector<std::string> names = {"model.embed_tokens.weight", "model.norm.weight", "lm_head.weight"};
    for (int l = 0; l < e->m.L; ++l)
      for (int k = 0; k < cruise::kLayerTensors; ++k)
        names.push_back("model.layers." + std::to_string(l) + "." + cruise::kLayerKeys[k]);
    for (const auto &n : names) {
      std::ifstream f(weights + "/" + n + ".bin", std::ios::binary | std::ios::ate);
      if (!f) { rc = -1; break; }
      std::vector<char> buf(static_cast<size_t>(f.tellg()));
      f.seekg(0, std::ios::beg);
      f.read(buf.data(), static_cast<std::streamsize>(buf.size()));
      if (!f || cruise::copy_tensor(e, n, buf.data(), buf.size(), true) != 0) { rc = -1; break; }
    }
  }
  if (rc != 0) {
    cruise::destroy_engine(e);
    *status = 4;
    cruise::g_create_error = "loading the weights from " + weights + " failed";
    return nullptr;
  }
  auto *be = new BridgeEngine();
  be->engine = e;
  cruise::g_bridge_active = true;
  *status = 0;
  return be;
}

int32_t resident_epoch_execute(void *opaque, int32_t request_count, int32_t max_steps,
                               const int64_t *input_token_ids, const int64_t *input_positions,
                               const int32_t *input_sequence_lengths, const int32_t *input_eos_token_ids,
                               const int32_t *input_row_generations, int64_t *output_token_ids,
                               int32_t *output_executed, int32_t *output_row_generations,
                               int32_t *output_model_calls, int32_t *output_device_status,
                               int32_t *output_feed_calls, int32_t *output_fetch_calls,
                               int32_t *output_commit_state, int32_t *output_kv_import_checksum,
                               int64_t *output_wall_us, int64_t *output_native_cpu_us,
                               int64_t *output_declared_input_bytes, int64_t *output_declared_output_bytes,
                               const char *transfer_path, uint64_t transfer_id,
                               const ResidentEpochIpcMetadata *ipc_metadata) {
  if (output_commit_state == nullptr) return 10;
  *output_commit_state = CRUISE_EPOCH_PREPARED;
  const bool device_import = ipc_metadata != nullptr;
  // no file and no IPC metadata but a transfer id: the rows resident_epoch_prefill computed
  const bool prefill_import = transfer_path == nullptr && !device_import && transfer_id != 0;
  const bool importing = transfer_path != nullptr || device_import || prefill_import;
  if (opaque == nullptr || request_count < 1 || request_count > kBatch || max_steps < 1 || max_steps > kMaxSteps ||
      input_token_ids == nullptr || input_positions == nullptr || input_sequence_lengths == nullptr ||
      input_eos_token_ids == nullptr || input_row_generations == nullptr || output_token_ids == nullptr ||
      output_executed == nullptr || output_row_generations == nullptr || output_model_calls == nullptr ||
      output_device_status == nullptr || output_feed_calls == nullptr || output_fetch_calls == nullptr ||
      output_kv_import_checksum == nullptr || output_wall_us == nullptr || output_native_cpu_us == nullptr ||
      output_declared_input_bytes == nullptr || output_declared_output_bytes == nullptr ||
      (importing && transfer_id == 0) || (!importing && transfer_id != 0) ||
      (transfer_path != nullptr && device_import))
    return 10;
  auto *be = static_cast<BridgeEngine *>(opaque);
  Engine *e = be->engine;
  std::lock_guard<std::mutex> lock(e->execute_mutex);
  cudaSetDevice(e->device);
  const cruise::ModelDims &m = e->m;
  std::vector<uint8_t> payload;
  int32_t import_mask = 0;
  uint32_t expected_checksum = 0;
  if (importing && !device_import && !prefill_import &&
      !cruise::read_transfer(e, transfer_path, transfer_id, input_row_generations, payload, import_mask,
                             expected_checksum))
    return 13;
  if (device_import) {
    // the IPC copy overwrites the staging buffer a pending prefill left
    be->prefill_mask = 0;
    e->payload_ready = false;
    if (!cruise::validate_ipc(e, ipc_metadata, input_row_generations) || !cruise::prepare_ipc_payload(be, ipc_metadata))
      return 35;
    import_mask = static_cast<int32_t>(ipc_metadata->import_mask);
  }
  if (prefill_import) {
    // every prefilled row is imported, and only into a row this epoch runs
    if (be->prefill_mask == 0 || !e->payload_ready) return 13;
    for (int r = 0; r < kBatch; ++r) {
      if (((be->prefill_mask >> r) & 1) == 0) continue;
      if (input_row_generations[r] == 0) return 13;
      if (input_positions[r] != be->prefill_lens[r] - 1) return 11;   // decodes from the last prompt token
    }
    import_mask = be->prefill_mask;
  }
  *output_model_calls = 0;
  *output_device_status = -1;
  *output_feed_calls = 0;
  *output_fetch_calls = 0;
  *output_kv_import_checksum = 0;
  *output_wall_us = 0;
  *output_native_cpu_us = 0;
  const int64_t payload_bytes = cruise::import_payload_bytes(e);
  *output_declared_input_bytes = device_import    ? CRUISE_SIDECAR_REQUEST_BYTES + CRUISE_RESIDENT_IPC_METADATA_BYTES
                                 : prefill_import ? 260
                                 : (importing ? payload_bytes + 244 : 260);
  *output_declared_output_bytes = 368;
  const int64_t cpu_start = cruise::process_cpu_us();
  std::fill(output_token_ids, output_token_ids + kBatch * kMaxSteps, -1);
  std::fill(output_executed, output_executed + kBatch, 0);
  std::fill(output_row_generations, output_row_generations + kBatch, 0);

  int64_t tokens[kBatch] = {0}, positions[kBatch] = {0};
  int32_t lengths[kBatch] = {0}, slots[kBatch] = {0}, active[kBatch] = {0};
  std::vector<int32_t> blocks(kBatch * m.bpr);
  for (int r = 0; r < kBatch; ++r)
    for (int j = 0; j < m.bpr; ++j) blocks[r * m.bpr + j] = r * m.bpr + j;   // :524-532
  auto slot_of = [&](int r, int64_t pos) {
    if (pos < 0 || pos >= m.C) return -1;
    return static_cast<int32_t>((r * m.bpr + pos / m.bs) * m.bs + pos % m.bs);
  };
  for (int r = 0; r < kBatch; ++r) slots[r] = slot_of(r, 0);
  int32_t count = 0;
  for (int r = 0; r < kBatch; ++r) {
    if (input_row_generations[r] == 0) continue;
    ++count;
    if (input_row_generations[r] < 0 || input_token_ids[r] < 0 || input_token_ids[r] >= m.V ||
        input_positions[r] < 0 || input_positions[r] + max_steps > m.C ||
        input_sequence_lengths[r] != input_positions[r] + 1 || input_eos_token_ids[r] < 0 ||
        input_eos_token_ids[r] >= m.V)
      return 11;
    tokens[r] = input_token_ids[r];
    positions[r] = input_positions[r];
    lengths[r] = input_sequence_lengths[r];
    slots[r] = slot_of(r, input_positions[r]);
    active[r] = 1;
  }
  if (count != request_count) return 12;
  int32_t control[cruise::kControlIn] = {0};
  control[0] = max_steps;
  for (int r = 0; r < kBatch; ++r)
    control[1 + r] = input_row_generations[r] != 0 ? input_eos_token_ids[r] : e->cfg.configured_eos;
  control[1 + kBatch] = 0;
  control[2 + kBatch] = importing ? (cruise::kImportFlag | import_mask) : 0;
  for (int r = 0; r < kBatch; ++r) control[3 + kBatch + r] = input_row_generations[r];

  int64_t history[kMaxSteps * kBatch];
  int32_t out[cruise::kControlOut];
  const auto wall_start = std::chrono::steady_clock::now();
  *output_commit_state = CRUISE_EPOCH_EXECUTING;
  // a prefill import passes no payload: run_epoch takes the prefilled device staging
  if (prefill_import) be->prefill_mask = 0;
  const int32_t rc = cruise::run_epoch(
      e, tokens, positions, lengths, slots, active, blocks.data(), e->tiling.data(), control,
      device_import ? static_cast<const void *>(e->d_payload) : (importing && !prefill_import ? payload.data() : nullptr),
      importing && !prefill_import ? static_cast<uint64_t>(payload_bytes) : 0, history, out, nullptr, nullptr,
      device_import);
  const auto wall_end = std::chrono::steady_clock::now();
  *output_feed_calls = 1;
  if (rc != 0) return 30;
  *output_fetch_calls = 1;
  *output_wall_us = std::chrono::duration_cast<std::chrono::microseconds>(wall_end - wall_start).count();
  *output_device_status = out[3];
  *output_model_calls = out[4];
  *output_kv_import_checksum = out[5];
  if (*output_device_status == 0) {
    if ((device_import || prefill_import) && *output_kv_import_checksum == 0) return 34;
    if (importing && !device_import && !prefill_import &&
        static_cast<uint32_t>(*output_kv_import_checksum) != expected_checksum)
      return 34;
  }
  for (int r = 0; r < kBatch; ++r) {
    const int32_t executed = out[6 + 2 * kBatch + r];
    if (executed < 0 || executed > max_steps) return 33;
    output_executed[r] = executed;
    output_row_generations[r] = out[6 + 4 * kBatch + 2 + r];
    for (int s = 0; s < executed; ++s) output_token_ids[r * kMaxSteps + s] = history[s * kBatch + r];
  }
  const int64_t cpu_end = cruise::process_cpu_us();
  if (cpu_start >= 0 && cpu_end >= cpu_start) *output_native_cpu_us = cpu_end - cpu_start;
  *output_commit_state = CRUISE_EPOCH_COMMITTED;
  return 0;
}

int32_t resident_epoch_prefill(void *opaque, const int64_t *prompt_tokens, const int32_t *prompt_lens,
                               int32_t stride) {
  if (opaque == nullptr || prompt_tokens == nullptr || prompt_lens == nullptr || stride < 1) return 10;
  auto *be = static_cast<BridgeEngine *>(opaque);
  Engine *e = be->engine;
  std::lock_guard<std::mutex> lock(e->execute_mutex);
  cudaSetDevice(e->device);
  be->prefill_mask = 0;
  int32_t mask = 0;
  for (int r = 0; r < kBatch; ++r) {
    if (prompt_lens[r] < 0 || prompt_lens[r] > stride) return 10;
    if (prompt_lens[r] >= 2) mask |= 1 << r;   // a 1-token prompt has no K/V before its decode position
  }
  if (mask == 0) return 10;
  const int32_t rc = cruise::prefill_run(e, prompt_tokens, prompt_lens, stride);
  if (rc == -1) return 11;   // a prompt longer than a block or a token outside the vocabulary
  if (rc != 0) return 30;
  be->prefill_mask = mask;
  for (int r = 0; r < kBatch; ++r) be->prefill_lens[r] = prompt_lens[r];
  return 0;
}

void resident_epoch_destroy(void *opaque) {
  if (opaque == nullptr) return;
  std::lock_guard<std::mutex> lifecycle(cruise::g_lifecycle_mutex);
  auto *be = static_cast<BridgeEngine *>(opaque);
  {
    std::lock_guard<std::mutex> lock(be->engine->execute_mutex);
    cudaSetDevice(be->engine->device);
    for (auto &entry : be->ipc_imports) cudaIpcCloseMemHandle(entry.second);
    be->ipc_imports.clear();
  }
  cruise::destroy_engine(be->engine);
  delete be;
  cruise::g_bridge_active = false;
}

}  // extern "C"
