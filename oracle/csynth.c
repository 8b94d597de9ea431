/*
 * csynth.c -- the seeded weight generator of oracle/synth.py in plain C with
 * OpenMP, for full-depth (28-layer, 15 GB) oracle models.  TEST
 * INFRASTRUCTURE ONLY: used by tests/ and by the CPU legs of bench.py, never
 * by the product.
 *
 * Element i of tensor t (seed s, standard deviation std):
 *   key   = mix(s * GAMMA + (t + 1) * KEYMUL)            (mod 2^64)
 *   h     = mix(key + (i + 1) * GAMMA)                   (mod 2^64)
 *   sum   = the four 16-bit lanes of h added             (Irwin-Hall(4))
 *   value = bf16_rne(float(2 * sum - 262140) * scale)    (one IEEE fp32 multiply)
 * mix is the splitmix64 finaliser (Steele, Lea, Flood, OOPSLA 2014).  Integer
 * arithmetic up to one correctly rounded multiply, so the bits equal
 * oracle/synth.py and the engine's device generator on any IEEE machine.
 */
#include <stdint.h>
#include <string.h>

#define GAMMA 0x9E3779B97F4A7C15ull
#define KEYMUL 0xD1B54A32D192ED03ull

static inline uint64_t mix(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

static inline uint16_t bf16_rne(float v) {
  uint32_t bits;
  memcpy(&bits, &v, 4);
  bits += 0x7FFFu + ((bits >> 16) & 1u);
  return (uint16_t)(bits >> 16);
}

/* Elements start .. start+count-1 of tensor `tensor_id` into out[0..count). */
void cruise_oracle_synth(uint64_t seed, int32_t tensor_id, int64_t start, int64_t count, float scale,
                         uint16_t *out, int32_t threads) {
  const uint64_t key = mix(seed * GAMMA + (uint64_t)(tensor_id + 1) * KEYMUL);
  if (threads < 1) threads = 1;
#pragma omp parallel for num_threads(threads) schedule(static)
  for (int64_t i = 0; i < count; ++i) {
    const uint64_t h = mix(key + (uint64_t)(start + i + 1) * GAMMA);
    const int32_t sum = (int32_t)((h & 0xFFFF) + ((h >> 16) & 0xFFFF) + ((h >> 32) & 0xFFFF) + (h >> 48));
    const float centred = (float)(2 * sum - 262140);
    out[i] = bf16_rne(centred * scale);
  }
}
