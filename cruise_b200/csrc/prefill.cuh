// Batched device prefill of a cohort's prompts (the path before the resident
// epoch): every prompt token of every row goes through the decoder layers at
// once, and each layer's roped K and V land in the import payload
// [K|V][layer][row][block_size][kv_heads][head_dim] -- the one-shot import
// format of the epoch controller -- at the token's position in its row's first
// block.  The projections run on the tensor cores (prefill_gemm.cuh, fp32
// accumulation and fp32 k-range partial sums, added in order here; the
// gate/up projection writes the SwiGLU activation itself).  These kernels do everything
// between them with the decoder step's rounding points
// (batched_decoder_step.py:224-229 norm, :305-313 QKV, :231-240 rope,
// :356-377 scores/softmax, :380-403 residuals and SwiGLU), token by token, so
// a prefilled token's K/V equal the single-token step's up to fp32 summation
// order.
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

// Programmatic dependent launch: the engine launches each prefill kernel so
// that it may begin while its predecessor in the stream drains.  A kernel
// first lets its own successor begin launching, then waits for the
// predecessor's completion (and its memory) before it reads or writes
// anything the predecessor touches.  Without the launch attribute both are no-ops.
__device__ __forceinline__ void chain_enter() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

// h[t] = embed[token[t]]; one CTA per token.
__global__ void embed_rows(const bf16 *embed, const int64_t *token, bf16 *h, int H) {
  chain_enter();
  const int t = blockIdx.x;
  const uint4 *src = reinterpret_cast<const uint4 *>(embed + token[t] * static_cast<int64_t>(H));
  uint4 *dst = reinterpret_cast<uint4 *>(h + static_cast<int64_t>(t) * H);
  for (int i = threadIdx.x; i < H / 8; i += blockDim.x) dst[i] = src[i];
}

// x[t] = bf16(bf16(h * rsqrt(mean(h^2) + eps)) * w): rms_norm (:224-229); one
// CTA per token.
__global__ void rms_norm_rows(const bf16 *h, const bf16 *w, bf16 *x, int H, float eps) {
  chain_enter();
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

// The residual update after the O and down projections followed by the next
// rms_norm, one CTA of kNormThreads per token.  hidden = residual +
// materialize(mm_t(x, W)) (:380-386, :399-403): h[t] = bf16(h + y), y the
// GEMM's fp32 sum already rounded to bf16 by the GEMM, added to the bf16
// residual, rounded again.  Then x[t] = bf16(bf16(h * rsqrt(mean(h^2) + eps)) *
// w).  Each thread owns chunks of 8 consecutive elements (16-byte loads of h,
// y and w), issues all its loads before the first store, and keeps the
// updated h in registers for the norm.  H % 8 == 0 and H <= 8 *
// kNormThreads * kNormChunks, both checked by the host.
constexpr int kNormThreads = 256;
constexpr int kNormChunks = 4;
constexpr int kMaxSplits = 8;   // k-range partial sums a consumer adds (the GEMM's split count is capped here)

__device__ __forceinline__ void unpack8(const uint4 &u, float (&v)[8]) {
  const __nv_bfloat162 *p = reinterpret_cast<const __nv_bfloat162 *>(&u);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    v[2 * k] = __low2float(p[k]);
    v[2 * k + 1] = __high2float(p[k]);
  }
}

__device__ __forceinline__ uint4 pack8(const float (&v)[8]) {
  uint4 u;
  uint32_t *w = reinterpret_cast<uint32_t *>(&u);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    __nv_bfloat162 pair = __floats2bfloat162_rn(v[2 * k], v[2 * k + 1]);
    w[k] = *reinterpret_cast<uint32_t *>(&pair);
  }
  return u;
}

__global__ void __launch_bounds__(kNormThreads) residual_rms_norm(const bf16 *y, bf16 *h, const bf16 *w, bf16 *x,
                                                                   int H, float eps) {
  chain_enter();
  __shared__ float scratch[32];
  const int64_t base = static_cast<int64_t>(blockIdx.x) * H;
  const int chunks = H >> 3;
  uint4 old[kNormChunks], sum[kNormChunks];
#pragma unroll
  for (int j = 0; j < kNormChunks; ++j) {
    const int c = threadIdx.x + j * kNormThreads;
    if (c < chunks) {
      old[j] = *reinterpret_cast<const uint4 *>(h + base + c * 8);
      sum[j] = *reinterpret_cast<const uint4 *>(y + base + c * 8);
    }
  }
  float hv[kNormChunks][8];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < kNormChunks; ++j) {
    const int c = threadIdx.x + j * kNormThreads;
    if (c < chunks) {
      float prev[8], a[8];
      unpack8(old[j], prev);
      unpack8(sum[j], a);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        hv[j][k] = r(__fadd_rn(prev[k], a[k]));
        ss = __fadd_rn(ss, __fmul_rn(hv[j][k], hv[j][k]));
      }
      *reinterpret_cast<uint4 *>(h + base + c * 8) = pack8(hv[j]);
    }
  }
  const float total = block_sum(ss, scratch);
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(total, static_cast<float>(H)), eps)));
#pragma unroll
  for (int j = 0; j < kNormChunks; ++j) {
    const int c = threadIdx.x + j * kNormThreads;
    if (c < chunks) {
      float wv[8], out[8];
      unpack8(*reinterpret_cast<const uint4 *>(w + c * 8), wv);
#pragma unroll
      for (int k = 0; k < 8; ++k) out[k] = __fmul_rn(r(__fmul_rn(hv[j][k], inv)), wv[k]);
      *reinterpret_cast<uint4 *>(x + base + c * 8) = pack8(out);
    }
  }
}

// The same residual update and norm from the projection's fp32 k-range
// partial sums [split][T][H] (tensor-core GEMM): y = bf16(sum of the splits in
// order) is the decoder's materialize(mm_t(x, W)), then h = bf16(h + y) and
// x = the next rms_norm, as above.  One CTA per token of H / 16 threads (two
// 8-element chunks each, so that 4 CTAs fit an SM and all tokens run in one
// wave); each round loads one split of both chunks.
constexpr int kPartsChunks = 2;

__host__ __device__ inline int parts_norm_threads(int H) { return ((H / 8 + kPartsChunks - 1) / kPartsChunks + 31) / 32 * 32; }

__global__ void __launch_bounds__(1024) residual_rms_norm_parts(const float *parts, int nsplit, int T, bf16 *h,
                                                                const bf16 *w, bf16 *x, int H, float eps) {
  chain_enter();
  __shared__ float scratch[32];
  const int64_t base = static_cast<int64_t>(blockIdx.x) * H;
  const int64_t split_stride = static_cast<int64_t>(T) * H;
  const int chunks = H >> 3;
  float acc[kPartsChunks][8];
  uint4 hraw[kPartsChunks];
#pragma unroll
  for (int j = 0; j < kPartsChunks; ++j) {
    const int c = threadIdx.x + j * blockDim.x;
    if (c < chunks) {
      hraw[j] = *reinterpret_cast<const uint4 *>(h + base + c * 8);
      const float4 *p0 = reinterpret_cast<const float4 *>(parts + base + c * 8);
      const float4 a = p0[0], b2 = p0[1];
      acc[j][0] = a.x; acc[j][1] = a.y; acc[j][2] = a.z; acc[j][3] = a.w;
      acc[j][4] = b2.x; acc[j][5] = b2.y; acc[j][6] = b2.z; acc[j][7] = b2.w;
    }
  }
  for (int k = 1; k < nsplit; ++k) {
    float4 lo[kPartsChunks], hi[kPartsChunks];
#pragma unroll
    for (int j = 0; j < kPartsChunks; ++j) {
      const int c = threadIdx.x + j * blockDim.x;
      if (c < chunks) {
        const float4 *pk = reinterpret_cast<const float4 *>(parts + k * split_stride + base + c * 8);
        lo[j] = pk[0];
        hi[j] = pk[1];
      }
    }
#pragma unroll
    for (int j = 0; j < kPartsChunks; ++j) {
      const int c = threadIdx.x + j * blockDim.x;
      if (c < chunks) {
        acc[j][0] = __fadd_rn(acc[j][0], lo[j].x); acc[j][1] = __fadd_rn(acc[j][1], lo[j].y);
        acc[j][2] = __fadd_rn(acc[j][2], lo[j].z); acc[j][3] = __fadd_rn(acc[j][3], lo[j].w);
        acc[j][4] = __fadd_rn(acc[j][4], hi[j].x); acc[j][5] = __fadd_rn(acc[j][5], hi[j].y);
        acc[j][6] = __fadd_rn(acc[j][6], hi[j].z); acc[j][7] = __fadd_rn(acc[j][7], hi[j].w);
      }
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < kPartsChunks; ++j) {
    const int c = threadIdx.x + j * blockDim.x;
    if (c < chunks) {
      float prev[8];
      unpack8(hraw[j], prev);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        acc[j][k] = r(__fadd_rn(prev[k], r(acc[j][k])));   // h + bf16(y), rounded
        ss = __fadd_rn(ss, __fmul_rn(acc[j][k], acc[j][k]));
      }
      *reinterpret_cast<uint4 *>(h + base + c * 8) = pack8(acc[j]);
    }
  }
  const float total = block_sum(ss, scratch);
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(total, static_cast<float>(H)), eps)));
#pragma unroll
  for (int j = 0; j < kPartsChunks; ++j) {
    const int c = threadIdx.x + j * blockDim.x;
    if (c < chunks) {
      float wv[8], out[8];
      unpack8(*reinterpret_cast<const uint4 *>(w + c * 8), wv);
#pragma unroll
      for (int k = 0; k < 8; ++k) out[k] = __fmul_rn(r(__fmul_rn(acc[j][k], inv)), wv[k]);
      *reinterpret_cast<uint4 *>(x + base + c * 8) = pack8(out);
    }
  }
}

// QKV epilogue, a row of CTAs per token (one unit per thread): q, k, v = bf16(acc + bias) (F.linear: fp32
// sum plus bias, one rounding), rope on q and k with the token's position
// (q*cos + rotate_half(q)*sin, each product and the sum rounded to bf16), q to
// `q_out` [T][Hq], k and v into the payload at (row, position).  A thread
// takes one unit: for q and k, the element pairs (i, i+1) of a head and their
// rotation partners (i+half, i+half+1), so each partner is loaded once; for v,
// two consecutive elements.  d is even and half = d/2 is even (d = 64 or 128).
__device__ __forceinline__ uint32_t bf2_bits(float lo, float hi) {
  __nv_bfloat162 pair = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&pair);
}

// The projection's fp32 sum of element n of this token: the k-range partial
// sums [split][T][N] added in split order (deterministic).
__device__ __forceinline__ float2 split_sum2(const float *acc, int64_t split_stride, int nsplit, int64_t at) {
  float2 v[kMaxSplits];   // every split's load in flight before the ordered sum
#pragma unroll
  for (int k = 0; k < kMaxSplits; ++k)
    if (k < nsplit) v[k] = *reinterpret_cast<const float2 *>(acc + k * split_stride + at);
  float2 s = v[0];
#pragma unroll
  for (int k = 1; k < kMaxSplits; ++k)
    if (k < nsplit) {
      s.x = __fadd_rn(s.x, v[k].x);
      s.y = __fadd_rn(s.y, v[k].y);
    }
  return s;
}

__global__ void qkv_rope_store(const float *acc, int nsplit, int T, const bf16 *bias, const bf16 *cos,
                               const bf16 *sin, const int32_t *tok_row, const int32_t *tok_pos, bf16 *q_out,
                               bf16 *payload, int layer, int L, int nq, int nkv, int d, int bs) {
  chain_enter();
  const int t = blockIdx.x;
  const int Hq = nq * d, kvw = nkv * d, N = Hq + 2 * kvw;
  const int row = tok_row[t], pos = tok_pos[t], half = d / 2, quarter = d / 4;
  const int64_t split_stride = static_cast<int64_t>(T) * N;
  const int64_t a = static_cast<int64_t>(t) * N;
  const bf16 *cs = cos + static_cast<int64_t>(pos) * d;
  const bf16 *sn = sin + static_cast<int64_t>(pos) * d;
  const int64_t block_elems = static_cast<int64_t>(bs) * kvw;
  const int64_t slot_off = (static_cast<int64_t>(layer) * kBatch + row) * block_elems + static_cast<int64_t>(pos) * kvw;
  const int64_t v_base = static_cast<int64_t>(L) * kBatch * block_elems;   // V half of the payload
  const int rope_units = (nq + nkv) * quarter, units = rope_units + kvw / 2;
  const int u = blockIdx.y * blockDim.x + threadIdx.x;   // one unit per thread
  if (u < units) {
    if (u >= rope_units) {   // v: two elements
      const int n = Hq + kvw + 2 * (u - rope_units);
      const float2 s2 = split_sum2(acc, split_stride, nsplit, a + n);
      const __nv_bfloat162 b2 = *reinterpret_cast<const __nv_bfloat162 *>(bias + n);
      *reinterpret_cast<uint32_t *>(payload + v_base + slot_off + (n - Hq - kvw)) =
          bf2_bits(__fadd_rn(s2.x, __low2float(b2)), __fadd_rn(s2.y, __high2float(b2)));
      return;
    }
    const int head = u / quarter, i = 2 * (u - head * quarter);   // q heads, then k heads
    const int n_lo = head * d + i, n_hi = n_lo + half;
    const float2 s_lo = split_sum2(acc, split_stride, nsplit, a + n_lo);
    const float2 s_hi = split_sum2(acc, split_stride, nsplit, a + n_hi);
    const __nv_bfloat162 b_lo = *reinterpret_cast<const __nv_bfloat162 *>(bias + n_lo);
    const __nv_bfloat162 b_hi = *reinterpret_cast<const __nv_bfloat162 *>(bias + n_hi);
    const __nv_bfloat162 c_lo = *reinterpret_cast<const __nv_bfloat162 *>(cs + i);
    const __nv_bfloat162 c_hi = *reinterpret_cast<const __nv_bfloat162 *>(cs + i + half);
    const __nv_bfloat162 z_lo = *reinterpret_cast<const __nv_bfloat162 *>(sn + i);
    const __nv_bfloat162 z_hi = *reinterpret_cast<const __nv_bfloat162 *>(sn + i + half);
    const float x0 = r(__fadd_rn(s_lo.x, __low2float(b_lo))), x1 = r(__fadd_rn(s_lo.y, __high2float(b_lo)));
    const float y0 = r(__fadd_rn(s_hi.x, __low2float(b_hi))), y1 = r(__fadd_rn(s_hi.y, __high2float(b_hi)));
    // rotate_half: element i pairs with -(i+half), element i+half with +(i)
    const float lo0 = r(__fadd_rn(r(__fmul_rn(x0, __low2float(c_lo))), r(__fmul_rn(-y0, __low2float(z_lo)))));
    const float lo1 = r(__fadd_rn(r(__fmul_rn(x1, __high2float(c_lo))), r(__fmul_rn(-y1, __high2float(z_lo)))));
    const float hi0 = r(__fadd_rn(r(__fmul_rn(y0, __low2float(c_hi))), r(__fmul_rn(x0, __low2float(z_hi)))));
    const float hi1 = r(__fadd_rn(r(__fmul_rn(y1, __high2float(c_hi))), r(__fmul_rn(x1, __high2float(z_hi)))));
    // a head lies wholly in q or wholly in k
    bf16 *dst = n_lo < Hq ? q_out + static_cast<int64_t>(t) * Hq + n_lo : payload + slot_off + (n_lo - Hq);
    *reinterpret_cast<uint32_t *>(dst) = bf2_bits(lo0, lo1);
    *reinterpret_cast<uint32_t *>(dst + half) = bf2_bits(hi0, hi1);
  }
}

// Tokens of the cohort in the order the host packs them: row by row, each
// row's positions 0..count-1 consecutive from `start`.
struct RowSpans {
  int32_t start[kBatch];
  int32_t count[kBatch];
};

constexpr int kAttnChunk = 16;     // query positions per CTA
constexpr int kAttnWarps = 16;     // 8 pairs; a pair takes 16 query rows
constexpr int kMaxKeys = 128;      // block_size bound: keys (and query rows) per CTA
constexpr int kAttnPairs = kAttnWarps / 2;
constexpr int kHalfKeys = kMaxKeys / 2;   // keys per warp of a pair in S = Q K^T

__host__ __device__ inline int attention_row_stride(int d) { return d + 8; }   // bf16; 16-byte pad per row

// Shared memory of causal_attention_mma: Q, K and V rows (kMaxKeys each,
// padded stride), each pair's bf16 probabilities P [16][kMaxKeys + 8], and the
// pairs' per-row partial maxima and sums.
__host__ __device__ inline int attention_p_stride() { return kMaxKeys + 8; }

__host__ __device__ inline size_t attention_smem_bytes(int bs, int d, int groups) {
  (void)bs;
  (void)groups;
  return static_cast<size_t>(3) * kMaxKeys * attention_row_stride(d) * 2 +
         static_cast<size_t>(kAttnPairs) * 16 * attention_p_stride() * 2 +
         static_cast<size_t>(2) * kAttnPairs * 2 * 16 * 4;
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// 16-byte asynchronous global -> shared copy; `src_bytes` 0 writes zeros and
// reads nothing.  Both addresses 16-byte aligned.
__device__ __forceinline__ void cp_async16(void *dst, const void *src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
               : "memory");
}

__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void *p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

__device__ __forceinline__ void ldsm_x2(uint32_t (&r)[2], const void *p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0, %1}, [%2];" : "=r"(r[0]), "=r"(r[1]) : "r"(smem_u32(p)));
}

__device__ __forceinline__ void ldsm_x2_trans(uint32_t (&r)[2], const void *p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0, %1}, [%2];"
               : "=r"(r[0]), "=r"(r[1])
               : "r"(smem_u32(p)));
}

// c += a (16x16 bf16, row) * b (16x8 bf16, col), fp32 accumulators
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t *>(&v);
}

// Causal attention of the query heads sharing one KV head, for a chunk of a
// row's prompt positions, on the tensor cores: grid (chunks, kv heads, rows),
// kAttnWarps warps in kAttnPairs pairs.  The chunk's query rows
// (position-major, head-minor) and the row's K and V up to the chunk's last
// position are staged in shared memory.  Pair p takes query rows
// [16p, 16p + 16):
//   S = Q K^T (m16n8k16 bf16 MMAs, fp32 sums), warp h of the pair over keys
//   [64h, 64h + 64) -> scores bf16(bf16(S) / sqrt(d)) with the causal mask
//   (:356-367) -> softmax in fp32 rounded to bf16 (:368-377): each warp's row
//   maxima and sums of exponentials meet through shared memory, so every
//   probability is exp(s - row max) / row sum over all the row's keys ->
//   P in shared memory -> O = P V, warp h of the pair over output dimensions
//   [h D/2, (h + 1) D/2) and all keys -> bf16(O).
// Every warp reaches every __syncthreads (pairs without rows skip the math).
// Requires block_size <= 128 and d in {64, 128}.
template <int D>
__global__ void __launch_bounds__(kAttnWarps * 32, 1) causal_attention_mma(
    const bf16 *q, const bf16 *payload, RowSpans spans, bf16 *out, int layer, int L, int nq, int nkv, int bs,
    float sqrt_d) {
  chain_enter();
  extern __shared__ __align__(16) uint8_t smem[];
  constexpr int S = D + 8;   // shared-memory row stride (bf16)
  constexpr int SP = kMaxKeys + 8;   // probability row stride (bf16)
  constexpr int DT = D / 16;         // output 8-column tiles per warp in O = P V
  const int chunk = blockIdx.x, kvh = blockIdx.y, row = blockIdx.z;
  const int count = spans.count[row];
  const int p0 = chunk * kAttnChunk;
  if (p0 >= count) return;   // uniform over the CTA
  const int p1 = min(count, p0 + kAttnChunk);   // positions [p0, p1) query keys [0, p1)
  const int groups = nq / nkv, kvw = nkv * D;
  const int rows = (p1 - p0) * groups;          // query rows of this CTA
  const int keys = (p1 + 15) & ~15;             // keys padded to the MMA k-step
  bf16 *qs = reinterpret_cast<bf16 *>(smem);
  bf16 *ks = qs + kMaxKeys * S;
  bf16 *vs = ks + kMaxKeys * S;
  bf16 *ps = vs + kMaxKeys * S;                                     // [pair][16][SP]
  float *red_max = reinterpret_cast<float *>(ps + kAttnPairs * 16 * SP);   // [pair][half][16]
  float *red_sum = red_max + kAttnPairs * 2 * 16;                   // [pair][half][16]
  const int64_t block_elems = static_cast<int64_t>(bs) * kvw;
  const bf16 *kg = payload + (static_cast<int64_t>(layer) * kBatch + row) * block_elems + kvh * D;
  const bf16 *vg = kg + static_cast<int64_t>(L) * kBatch * block_elems;
  // stage K / V rows [0, keys) (zero beyond p1) and Q rows [0, 16 * ceil(rows / 16)) (zero beyond rows):
  // every copy of the thread is issued before the one wait
  constexpr int U = D / 8;   // 16-byte units per row
  for (int i = threadIdx.x; i < keys * U; i += blockDim.x) {
    const int j = i / U, u = i % U;
    const int64_t off = j < p1 ? static_cast<int64_t>(j) * kvw + u * 8 : 0;
    cp_async16(ks + j * S + u * 8, kg + off, j < p1 ? 16 : 0);
    cp_async16(vs + j * S + u * 8, vg + off, j < p1 ? 16 : 0);
  }
  const int qrows = (rows + 15) & ~15;
  const bf16 *q_first = q + static_cast<int64_t>(spans.start[row] + p0) * nq * D + kvh * groups * D;
  for (int i = threadIdx.x; i < qrows * U; i += blockDim.x) {
    const int r = i / U, u = i % U;
    const bf16 *src = q_first;
    if (r < rows) {
      const int t = spans.start[row] + p0 + r / groups, h = kvh * groups + r % groups;
      src = q + static_cast<int64_t>(t) * nq * D + h * D + u * 8;
    }
    cp_async16(qs + r * S + u * 8, src, r < rows ? 16 : 0);
  }
  cp_async_wait_all();
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int pair = warp >> 1, half = warp & 1;
  const int m0 = pair * 16;
  const bool busy = m0 < rows;
  const int g = lane >> 2, tq = lane & 3;
  const int rA = m0 + g, rB = rA + 8;
  const int posA = rA < rows ? p0 + rA / groups : -1, posB = rB < rows ? p0 + rB / groups : -1;
  const int ntiles = keys / 8;           // 8-key tiles holding keys
  const int nt0 = half * (kHalfKeys / 8);  // this warp's first key tile
  // S = Q K^T over this warp's 64 keys (8 n-tiles of 8)
  float sc[kHalfKeys / 8][4];
#pragma unroll
  for (int nt = 0; nt < kHalfKeys / 8; ++nt) sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
  if (busy) {
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      uint32_t a[4];
      ldsm_x4(a, qs + (m0 + (lane & 15)) * S + kk * 16 + (lane >> 4) * 8);
#pragma unroll
      for (int nt = 0; nt < kHalfKeys / 8; ++nt) {
        if (nt0 + nt < ntiles) {
          uint32_t bfrag[2];
          ldsm_x2(bfrag, ks + ((nt0 + nt) * 8 + (lane & 7)) * S + kk * 16 + ((lane >> 3) & 1) * 8);
          mma16816(sc[nt], a, bfrag);
        }
      }
    }
  }
  // scores and causal mask; this warp's row maxima
  float mxA = -INFINITY, mxB = -INFINITY;
#pragma unroll
  for (int nt = 0; nt < kHalfKeys / 8; ++nt) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int key = (nt0 + nt) * 8 + tq * 2 + j;
      const bool inA = nt0 + nt < ntiles && key <= posA, inB = nt0 + nt < ntiles && key <= posB;
      sc[nt][j] = inA ? r(__fdiv_rn(r(sc[nt][j]), sqrt_d)) : -INFINITY;
      sc[nt][2 + j] = inB ? r(__fdiv_rn(r(sc[nt][2 + j]), sqrt_d)) : -INFINITY;
      mxA = fmaxf(mxA, sc[nt][j]);
      mxB = fmaxf(mxB, sc[nt][2 + j]);
    }
  }
  mxA = fmaxf(mxA, __shfl_xor_sync(0xffffffffu, mxA, 1));
  mxA = fmaxf(mxA, __shfl_xor_sync(0xffffffffu, mxA, 2));
  mxB = fmaxf(mxB, __shfl_xor_sync(0xffffffffu, mxB, 1));
  mxB = fmaxf(mxB, __shfl_xor_sync(0xffffffffu, mxB, 2));
  float *my_max = red_max + (pair * 2 + half) * 16, *my_sum = red_sum + (pair * 2 + half) * 16;
  const float *other_max = red_max + (pair * 2 + (half ^ 1)) * 16;
  const float *other_sum = red_sum + (pair * 2 + (half ^ 1)) * 16;
  if (tq == 0) {
    my_max[g] = mxA;
    my_max[g + 8] = mxB;
  }
  __syncthreads();
  // the row maximum over all keys (max is exact in any order)
  mxA = fmaxf(mxA, other_max[g]);
  mxB = fmaxf(mxB, other_max[g + 8]);
  if (posA < 0) mxA = 0.f;   // padding rows: no keys, all probabilities 0
  if (posB < 0) mxB = 0.f;
  float sumA = 0.f, sumB = 0.f;
#pragma unroll
  for (int nt = 0; nt < kHalfKeys / 8; ++nt) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      sc[nt][j] = sc[nt][j] == -INFINITY ? 0.f : expf(__fsub_rn(sc[nt][j], mxA));
      sc[nt][2 + j] = sc[nt][2 + j] == -INFINITY ? 0.f : expf(__fsub_rn(sc[nt][2 + j], mxB));
      sumA += sc[nt][j];
      sumB += sc[nt][2 + j];
    }
  }
  sumA += __shfl_xor_sync(0xffffffffu, sumA, 1);
  sumA += __shfl_xor_sync(0xffffffffu, sumA, 2);
  sumB += __shfl_xor_sync(0xffffffffu, sumB, 1);
  sumB += __shfl_xor_sync(0xffffffffu, sumB, 2);
  if (tq == 0) {
    my_sum[g] = sumA;
    my_sum[g + 8] = sumB;
  }
  __syncthreads();
  // both halves in the same order on both warps: keys [0, 64) then [64, 128)
  {
    const float lowA = half == 0 ? sumA : other_sum[g], highA = half == 0 ? other_sum[g] : sumA;
    const float lowB = half == 0 ? sumB : other_sum[g + 8], highB = half == 0 ? other_sum[g + 8] : sumB;
    sumA = lowA + highA;
    sumB = lowB + highB;
  }
  if (posA < 0) sumA = 1.f;
  if (posB < 0) sumB = 1.f;
  // P = bf16(e / sum) into the pair's probability rows (this warp's keys)
  bf16 *prow = ps + pair * 16 * SP;
#pragma unroll
  for (int nt = 0; nt < kHalfKeys / 8; ++nt) {
    if (busy && nt0 + nt < ntiles) {
      const int key = (nt0 + nt) * 8 + tq * 2;
      *reinterpret_cast<uint32_t *>(prow + g * SP + key) =
          pack_bf16(r(__fdiv_rn(sc[nt][0], sumA)), r(__fdiv_rn(sc[nt][1], sumA)));
      *reinterpret_cast<uint32_t *>(prow + (g + 8) * SP + key) =
          pack_bf16(r(__fdiv_rn(sc[nt][2], sumB)), r(__fdiv_rn(sc[nt][3], sumB)));
    }
  }
  __syncthreads();
  if (!busy) return;
  // O = P V over all keys, this warp's output columns [half * D / 2, (half + 1) * D / 2)
  float o[DT][4];
#pragma unroll
  for (int nt = 0; nt < DT; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.f;
  const int dt0 = half * DT;
#pragma unroll
  for (int kj = 0; kj < kMaxKeys / 16; ++kj) {
    if (kj * 16 < keys) {
      uint32_t a[4];
      ldsm_x4(a, prow + (lane & 15) * SP + kj * 16 + (lane >> 4) * 8);
#pragma unroll
      for (int nt = 0; nt < DT; ++nt) {
        uint32_t bfrag[2];
        ldsm_x2_trans(bfrag, vs + (kj * 16 + (lane & 7) + ((lane >> 3) & 1) * 8) * S + (dt0 + nt) * 8);
        mma16816(o[nt], a, bfrag);
      }
    }
  }
  // bf16(O) to the token's head slice
  const int64_t tA = spans.start[row] + posA, tB = spans.start[row] + posB;
  const int hA = kvh * groups + rA % groups, hB = kvh * groups + rB % groups;
#pragma unroll
  for (int nt = 0; nt < DT; ++nt) {
    const int dim = (dt0 + nt) * 8 + tq * 2;
    if (posA >= 0)
      *reinterpret_cast<__nv_bfloat162 *>(out + tA * nq * D + hA * D + dim) = __floats2bfloat162_rn(o[nt][0], o[nt][1]);
    if (posB >= 0)
      *reinterpret_cast<__nv_bfloat162 *>(out + tB * nq * D + hB * D + dim) = __floats2bfloat162_rn(o[nt][2], o[nt][3]);
  }
}

}  // namespace prefill
}  // namespace cruise
