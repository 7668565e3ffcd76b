/*
 * Seeded synthetic weight generator for .yalm checkpoints (host code, no GPU).
 *
 * Element i of a tensor drawn with (seed, stream) is a deterministic function of those three
 * numbers only, so the contents do not depend on the number of threads or on the order in which
 * tensors are written.  Normal deviates come from the Box-Muller transform of two 32-bit uniforms
 * taken from one splitmix64 output per element pair.
 */
#include <math.h>
#include <omp.h>
#include <stdint.h>
#include <string.h>

/* Thread count for the fills (launchers such as torchrun set OMP_NUM_THREADS=1 per process, which
 * would make a 7B checkpoint take minutes to generate). */
void synth_set_threads(int n) {
  if (n > 0) omp_set_num_threads(n);
}

static inline uint64_t splitmix64(uint64_t z) {
  z += 0x9e3779b97f4a7c15ull;
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}

static inline uint16_t f32_to_f16_rne(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t absx = x & 0x7fffffffu;
  if (absx >= 0x7f800000u) return (uint16_t)(sign | 0x7c00u | (absx > 0x7f800000u ? 0x200u : 0));
  if (absx >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);
  if (absx < 0x38800000u) {
    if (absx < 0x33000000u) return (uint16_t)sign;
    uint32_t e = absx >> 23, m = (absx & 0x7fffffu) | 0x800000u, sh = 126u - e;
    uint32_t q = m >> sh, rem = m & ((1u << sh) - 1u), half = 1u << (sh - 1u);
    if (rem > half || (rem == half && (q & 1u))) q++;
    return (uint16_t)(sign | q);
  }
  uint32_t q = (((absx >> 23) - 112u) << 10) | ((absx & 0x7fffffu) >> 13);
  uint32_t rem = absx & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) q++;
  return (uint16_t)(sign | q);
}

/* Writes n fp16 values std * N(0,1) for (seed, stream) into out. */
void synth_fill_normal_f16(uint16_t* out, int64_t n, uint64_t seed, uint64_t stream, float std) {
  const uint64_t key = splitmix64(seed * 0x2545f4914f6cdd1dull ^ splitmix64(stream + 0x632be59bd9b4e019ull));
  const int64_t pairs = (n + 1) / 2;
  int64_t p;
#pragma omp parallel for schedule(static)
  for (p = 0; p < pairs; ++p) {
    uint64_t r = splitmix64(key + (uint64_t)p);
    /* u1 in (0,1], u2 in [0,1) */
    double u1 = ((double)(uint32_t)(r >> 32) + 1.0) * (1.0 / 4294967296.0);
    double u2 = (double)(uint32_t)r * (1.0 / 4294967296.0);
    double rad = sqrt(-2.0 * log(u1));
    double ang = 6.283185307179586 * u2;
    float z0 = (float)(rad * cos(ang)) * std;
    float z1 = (float)(rad * sin(ang)) * std;
    out[2 * p] = f32_to_f16_rne(z0);
    if (2 * p + 1 < n) out[2 * p + 1] = f32_to_f16_rne(z1);
  }
}

/* Writes n fp8 E5M2 values: each is the fp16 value synth_fill_normal_f16 would write for the same
 * (seed, stream, element), rounded to nearest even on its top byte (an E5M2 value is the top byte
 * of the fp16 with the same value). */
void synth_fill_normal_e5m2(uint8_t* out, int64_t n, uint64_t seed, uint64_t stream, float std) {
  const uint64_t key = splitmix64(seed * 0x2545f4914f6cdd1dull ^ splitmix64(stream + 0x632be59bd9b4e019ull));
  const int64_t pairs = (n + 1) / 2;
  int64_t p;
#pragma omp parallel for schedule(static)
  for (p = 0; p < pairs; ++p) {
    uint64_t r = splitmix64(key + (uint64_t)p);
    double u1 = ((double)(uint32_t)(r >> 32) + 1.0) * (1.0 / 4294967296.0);
    double u2 = (double)(uint32_t)r * (1.0 / 4294967296.0);
    double rad = sqrt(-2.0 * log(u1));
    double ang = 6.283185307179586 * u2;
    uint16_t h[2] = {f32_to_f16_rne((float)(rad * cos(ang)) * std), f32_to_f16_rne((float)(rad * sin(ang)) * std)};
    for (int j = 0; j < 2; ++j) {
      if (2 * p + j >= n) break;
      uint32_t lo = h[j] & 0xFFu, up = h[j] >> 8;
      if ((h[j] & 0x7FFFu) > 0x7C00u) {
        up |= 0x02u; /* NaN stays NaN */
      } else if (lo > 0x80u || (lo == 0x80u && (up & 1u))) {
        up += 1u;
      }
      out[2 * p + j] = (uint8_t)up;
    }
  }
}

/* Writes n fp32 copies of value (norm weights). */
void synth_fill_const_f32(float* out, int64_t n, float value) {
  int64_t i;
#pragma omp parallel for schedule(static)
  for (i = 0; i < n; ++i) out[i] = value;
}
