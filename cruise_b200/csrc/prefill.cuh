// Batched device prefill of a cohort's prompts (the path before the resident
// epoch): every prompt token of every row goes through the decoder layers at
// once, and each layer's roped K and V land in the import payload
// [K|V][layer][row][block_size][kv_heads][head_dim] -- the one-shot import
// format of the epoch controller -- at the token's position in its row's first
// block.  The projections are plain row-major bf16 GEMMs (cuBLAS, fp32
// accumulation, fp32 output); these kernels do everything between them with
// the decoder step's rounding points (batched_decoder_step.py:224-229 norm,
// :305-313 QKV, :231-240 rope, :356-377 scores/softmax, :380-403 residuals and
// SwiGLU), token by token, so a prefilled token's K/V equal the single-token
// step's up to fp32 summation order.
#pragma once

#include <cuda_bf16.h>
#include <cstdint>

#include "epoch_types.h"

namespace cruise {
namespace prefill {

using bf16 = __nv_bfloat16;

__device__ __forceinline__ float f(bf16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float r(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }
__device__ __forceinline__ bf16 b(float v) { return __float2bfloat16_rn(v); }

// Block-wide sum / max for blockDim.x a multiple of 32 (<= 1024); `scratch`
// holds 32 floats.  Every thread gets the result.
__device__ __forceinline__ float block_sum(float v, float *scratch) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) scratch[w] = v;
  __syncthreads();
  float t = 0.f;
  for (int i = 0; i < nw; ++i) t += scratch[i];
  return t;
}

__device__ __forceinline__ float block_max(float v, float *scratch) {
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) scratch[w] = v;
  __syncthreads();
  float t = scratch[0];
  for (int i = 1; i < nw; ++i) t = fmaxf(t, scratch[i]);
  return t;
}

// h[t] = embed[token[t]]; one CTA per token.
__global__ void embed_rows(const bf16 *embed, const int64_t *token, bf16 *h, int H) {
  const int t = blockIdx.x;
  const uint4 *src = reinterpret_cast<const uint4 *>(embed + token[t] * static_cast<int64_t>(H));
  uint4 *dst = reinterpret_cast<uint4 *>(h + static_cast<int64_t>(t) * H);
  for (int i = threadIdx.x; i < H / 8; i += blockDim.x) dst[i] = src[i];
}

// x[t] = bf16(bf16(h * rsqrt(mean(h^2) + eps)) * w): rms_norm (:224-229); one
// CTA per token.
__global__ void rms_norm_rows(const bf16 *h, const bf16 *w, bf16 *x, int H, float eps) {
  __shared__ float scratch[32];
  const bf16 *row = h + static_cast<int64_t>(blockIdx.x) * H;
  float ss = 0.f;
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    const float v = f(row[i]);
    ss = __fadd_rn(ss, __fmul_rn(v, v));
  }
  const float total = block_sum(ss, scratch);
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(total, static_cast<float>(H)), eps)));
  bf16 *out = x + static_cast<int64_t>(blockIdx.x) * H;
  for (int i = threadIdx.x; i < H; i += blockDim.x) out[i] = b(__fmul_rn(r(__fmul_rn(f(row[i]), inv)), f(w[i])));
}

// QKV epilogue, one CTA per token: q, k, v = bf16(acc + bias) (F.linear: fp32
// sum plus bias, one rounding), rope on q and k with the token's position
// (q*cos + rotate_half(q)*sin, each product and the sum rounded to bf16), q to
// `q_out` [T][Hq], k and v into the payload at (row, position).
__global__ void qkv_rope_store(const float *acc, const bf16 *bias, const bf16 *cos, const bf16 *sin,
                               const int32_t *tok_row, const int32_t *tok_pos, bf16 *q_out, bf16 *payload,
                               int layer, int L, int nq, int nkv, int d, int bs) {
  const int t = blockIdx.x;
  const int Hq = nq * d, kvw = nkv * d, N = Hq + 2 * kvw;
  const int row = tok_row[t], pos = tok_pos[t], half = d / 2;
  const float *a = acc + static_cast<int64_t>(t) * N;
  const bf16 *cs = cos + static_cast<int64_t>(pos) * d;
  const bf16 *sn = sin + static_cast<int64_t>(pos) * d;
  const int64_t block_elems = static_cast<int64_t>(bs) * kvw;
  const int64_t slot_off = (static_cast<int64_t>(layer) * kBatch + row) * block_elems + static_cast<int64_t>(pos) * kvw;
  const int64_t v_base = static_cast<int64_t>(L) * kBatch * block_elems;   // V half of the payload
  for (int n = threadIdx.x; n < N; n += blockDim.x) {
    const float x = r(__fadd_rn(a[n], f(bias[n])));
    if (n >= Hq + kvw) {   // v
      payload[v_base + slot_off + (n - Hq - kvw)] = b(x);
      continue;
    }
    const int base = n - n % d, i = n % d;
    const int pn = base + (i < half ? i + half : i - half);
    const float partner = r(__fadd_rn(a[pn], f(bias[pn])));
    const float rot = i < half ? -partner : partner;
    const float roped = r(__fadd_rn(r(__fmul_rn(x, f(cs[i]))), r(__fmul_rn(rot, f(sn[i])))));
    if (n < Hq) {
      q_out[static_cast<int64_t>(t) * Hq + n] = b(roped);
    } else {
      payload[slot_off + (n - Hq)] = b(roped);
    }
  }
}

// Tokens of the cohort in the order the host packs them: row by row, each
// row's positions 0..count-1 consecutive from `start`.
struct RowSpans {
  int32_t start[kBatch];
  int32_t count[kBatch];
};

constexpr int kAttnChunk = 16;     // query positions per CTA
constexpr int kAttnWarps = 8;
constexpr int kKeyStride = 130;    // bf16 per staged K row: 65 words, so 32 lanes reading 32 keys hit 32 banks

__host__ __device__ inline size_t attention_smem_bytes(int bs, int d, int groups) {
  return static_cast<size_t>(bs) * kKeyStride * 2 + static_cast<size_t>(bs) * d * 2 +
         static_cast<size_t>(kAttnChunk) * groups * d * 4 + static_cast<size_t>(kAttnWarps) * bs * 4;
}

// Causal attention of the query heads sharing one KV head, for a chunk of a
// row's prompt positions: grid (chunks, kv heads, rows), kAttnWarps warps.
// The row's K and V up to the chunk's last position are staged in shared
// memory once and read by every (position, head) pair of the chunk; a warp
// takes one pair at a time: scores bf16(bf16(q.k) / sqrt(d)) with a lane per
// key (:356-367), softmax in fp32 rounded to bf16 (:368-377), then
// bf16(sum_j p_j v_j) with a lane per d/32 dims, positions ascending.
// Requires block_size <= 128 and d a multiple of 32, d <= 128.
__global__ void causal_attention(const bf16 *q, const bf16 *payload, RowSpans spans, bf16 *out, int layer, int L,
                                 int nq, int nkv, int d, int bs, float sqrt_d) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int chunk = blockIdx.x, kvh = blockIdx.y, row = blockIdx.z;
  const int count = spans.count[row];
  const int p0 = chunk * kAttnChunk;
  if (p0 >= count) return;
  const int p1 = min(count, p0 + kAttnChunk);   // positions [p0, p1)
  const int groups = nq / nkv, kvw = nkv * d;
  bf16 *ks = reinterpret_cast<bf16 *>(smem);
  bf16 *vs = ks + static_cast<size_t>(bs) * kKeyStride;
  float *qs = reinterpret_cast<float *>(vs + static_cast<size_t>(bs) * d);
  float *ps = qs + static_cast<size_t>(kAttnChunk) * groups * d;
  const int64_t block_elems = static_cast<int64_t>(bs) * kvw;
  const bf16 *kg = payload + (static_cast<int64_t>(layer) * kBatch + row) * block_elems + kvh * d;
  const bf16 *vg = kg + static_cast<int64_t>(L) * kBatch * block_elems;
  // stage K and V of positions 0..p1-1 (2-element words) and the chunk's queries
  const int half_d = d / 2;
  for (int i = threadIdx.x; i < p1 * half_d; i += blockDim.x) {
    const int j = i / half_d, w = i % half_d;
    reinterpret_cast<uint32_t *>(ks + static_cast<size_t>(j) * kKeyStride)[w] =
        reinterpret_cast<const uint32_t *>(kg + static_cast<int64_t>(j) * kvw)[w];
    reinterpret_cast<uint32_t *>(vs + static_cast<size_t>(j) * d)[w] =
        reinterpret_cast<const uint32_t *>(vg + static_cast<int64_t>(j) * kvw)[w];
  }
  const int pairs = (p1 - p0) * groups;
  for (int i = threadIdx.x; i < pairs * d; i += blockDim.x) {
    const int pair = i / d, k = i % d;
    const int t = spans.start[row] + p0 + pair / groups, h = kvh * groups + pair % groups;
    qs[i] = f(q[static_cast<int64_t>(t) * nq * d + h * d + k]);
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float *pw = ps + static_cast<size_t>(warp) * bs;
  const int dims = d / 32;
  for (int pair = warp; pair < pairs; pair += kAttnWarps) {
    const int pos = p0 + pair / groups, h = kvh * groups + pair % groups;
    const int n = pos + 1;   // keys 0..pos
    const float *qv = qs + static_cast<size_t>(pair) * d;
    float sc[4], mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int j = lane + 32 * i;
      sc[i] = -INFINITY;
      if (j < n) {
        const uint32_t *kr = reinterpret_cast<const uint32_t *>(ks + static_cast<size_t>(j) * kKeyStride);
        float dot = 0.f;
        for (int w = 0; w < half_d; ++w) {
          const __nv_bfloat162 k2 = *reinterpret_cast<const __nv_bfloat162 *>(kr + w);
          dot = fmaf(qv[2 * w], __low2float(k2), dot);
          dot = fmaf(qv[2 * w + 1], __high2float(k2), dot);
        }
        sc[i] = r(__fdiv_rn(r(dot), sqrt_d));
        mx = fmaxf(mx, sc[i]);
      }
    }
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float e[4], sum = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      e[i] = lane + 32 * i < n ? expf(__fsub_rn(sc[i], mx)) : 0.f;
      sum += e[i];
    }
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
#pragma unroll
    for (int i = 0; i < 4; ++i)
      if (lane + 32 * i < n) pw[lane + 32 * i] = r(__fdiv_rn(e[i], sum));
    __syncwarp();
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int j = 0; j < n; ++j) {
      const float pj = pw[j];
      const bf16 *vr = vs + static_cast<size_t>(j) * d + lane * dims;
#pragma unroll
      for (int c = 0; c < 4; ++c)
        if (c < dims) acc[c] = fmaf(pj, f(vr[c]), acc[c]);
    }
    bf16 *dst = out + static_cast<int64_t>(spans.start[row] + pos) * nq * d + h * d + lane * dims;
#pragma unroll
    for (int c = 0; c < 4; ++c)
      if (c < dims) dst[c] = b(acc[c]);
    __syncwarp();
  }
}

// hidden = residual + materialize(mm_t(x, W)) (:380-386, :399-403): the GEMM's
// fp32 sum rounded to bf16, added to the bf16 residual, rounded again.
__global__ void add_residual(const float *acc, bf16 *h, int64_t count) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < count;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    h[i] = b(__fadd_rn(f(h[i]), r(acc[i])));
}

// silu(bf16(x Wg^T)) * bf16(x Wu^T), each op rounded to bf16 (:391-398); acc
// rows are [gate (I) | up (I)] per token.
__global__ void swiglu(const float *acc, bf16 *act, int T, int I) {
  const int64_t count = static_cast<int64_t>(T) * I;
  for (int64_t e = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; e < count;
       e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t t = e / I, i = e % I;
    const float gate = r(acc[t * 2 * I + i]);
    const float up = r(acc[t * 2 * I + I + i]);
    const float silu = r(__fdiv_rn(gate, __fadd_rn(1.0f, expf(-gate))));
    act[e] = b(__fmul_rn(silu, up));
  }
}

}  // namespace prefill
}  // namespace cruise
