/*
 * TEST INFRASTRUCTURE ONLY.  CPU restatement of GdsLLM's dequantization
 * formulas, used as the parity checker by tests/, __graft_entry__.smoke() and
 * the cpu_baseline leg of bench.py.  The product never calls this file.
 *
 *   Q4_0    gdsllm/runtime/gguf_dequant.cu:96-107
 *           out[j]    = fp16( f32(d) * f32((qs[j] & 15) - 8) )
 *           out[j+16] = fp16( f32(d) * f32((qs[j] >> 4) - 8) )
 *   Q8_0    gdsllm/runtime/gguf_dequant.cu:52-57
 *           out[i] = fp16( f32(d) * f32(qs[i]) )
 *   affine  gdsllm/runtime/affine_q4_dequant.cu:54-56 (and :113-115 in the
 *           fused kernel): out = fp16( nibble * scale + bias ) in fp32.  The
 *           product of a 4-bit integer and an fp16 scale is exact in fp32,
 *           so the value is rounded exactly once (at the add) whether or not
 *           nvcc contracts it to an FMA; fmaf states that single rounding.
 *
 * fp16 <-> fp32 conversions are written out here (IEEE 754 binary16,
 * round-to-nearest-even), not taken from a library.
 * Loops over independent blocks are split across OpenMP threads.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

float gdsq_oracle_half_to_float(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1Fu;
  uint32_t man = h & 0x3FFu;
  uint32_t bits;
  if (exp == 0x1Fu) {
    bits = sign | 0x7F800000u | (man << 13);
  } else if (exp != 0) {
    bits = sign | ((exp + 112u) << 23) | (man << 13);
  } else if (man == 0) {
    bits = sign;
  } else {
    /* subnormal: normalise */
    int e = -1;
    do {
      man <<= 1;
      ++e;
    } while ((man & 0x400u) == 0);
    man &= 0x3FFu;
    bits = sign | ((uint32_t)(112 - e) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

uint16_t gdsq_oracle_float_to_half(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  const uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
  const uint32_t ax = x & 0x7FFFFFFFu;
  if (ax >= 0x7F800000u) { /* inf / nan */
    if (ax == 0x7F800000u) return sign | 0x7C00u;
    return sign | 0x7E00u | (uint16_t)((ax >> 13) & 0x1FFu);
  }
  if (ax >= 0x477FF000u) return sign | 0x7C00u; /* >= 65520 rounds to inf */
  if (ax >= 0x38800000u) {                       /* normal fp16 range */
    const uint32_t r = ax - 0x38000000u;         /* rebias 127 -> 15 */
    return sign | (uint16_t)((r + 0xFFFu + ((r >> 13) & 1u)) >> 13);
  }
  if (ax < 0x33000000u) return sign; /* below half the smallest subnormal */
  /* subnormal result: k * 2^-24 with k = RNE(value * 2^24) */
  const uint32_t e = ax >> 23;
  const uint32_t m = (ax & 0x7FFFFFu) | 0x800000u;
  const uint32_t shift = 126u - e; /* 14..24 */
  uint32_t k = m >> shift;
  const uint32_t rem = m & ((1u << shift) - 1u);
  const uint32_t halfway = 1u << (shift - 1u);
  if (rem > halfway || (rem == halfway && (k & 1u))) ++k;
  return sign | (uint16_t)k;
}

static uint16_t load_u16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

void gdsq_oracle_dequant_q4_0(const uint8_t* src, uint16_t* dst, uint64_t num_blocks) {
  int64_t nb = (int64_t)num_blocks;
#pragma omp parallel for schedule(static)
  for (int64_t b = 0; b < nb; ++b) {
    const uint8_t* blk = src + b * 18;
    const float d = gdsq_oracle_half_to_float(load_u16(blk));
    const uint8_t* qs = blk + 2;
    uint16_t* out = dst + b * 32;
    for (int j = 0; j < 16; ++j) {
      const int lo = qs[j] & 0x0F;
      const int hi = qs[j] >> 4;
      out[j] = gdsq_oracle_float_to_half(d * (float)(lo - 8));
      out[j + 16] = gdsq_oracle_float_to_half(d * (float)(hi - 8));
    }
  }
}

void gdsq_oracle_dequant_q8_0(const uint8_t* src, uint16_t* dst, uint64_t num_blocks) {
  int64_t nb = (int64_t)num_blocks;
#pragma omp parallel for schedule(static)
  for (int64_t b = 0; b < nb; ++b) {
    const uint8_t* blk = src + b * 34;
    const float d = gdsq_oracle_half_to_float(load_u16(blk));
    const int8_t* qs = (const int8_t*)(blk + 2);
    uint16_t* out = dst + b * 32;
    for (int i = 0; i < 32; ++i) out[i] = gdsq_oracle_float_to_half(d * (float)qs[i]);
  }
}

/* weight: num_elements/8 words; scales/biases: num_elements/group_size. */
void gdsq_oracle_dequant_affine_q4(const uint32_t* weight, const uint16_t* scales,
                                   const uint16_t* biases, uint16_t* dst, uint64_t num_elements,
                                   int group_size) {
  const int64_t groups = (int64_t)(num_elements / (uint64_t)group_size);
  const int words_per_group = group_size / 8;
#pragma omp parallel for schedule(static)
  for (int64_t g = 0; g < groups; ++g) {
    const float s = gdsq_oracle_half_to_float(scales[g]);
    const float bias = gdsq_oracle_half_to_float(biases[g]);
    const uint32_t* w = weight + g * words_per_group;
    uint16_t* out = dst + g * group_size;
    for (int wi = 0; wi < words_per_group; ++wi) {
      const uint32_t packed = w[wi];
      for (int n = 0; n < 8; ++n) {
        const float nib = (float)((packed >> (4 * n)) & 0xFu);
        out[wi * 8 + n] = gdsq_oracle_float_to_half(fmaf(nib, s, bias));
      }
    }
  }
}

/* Bulk fp16 <-> fp32 conversion (used to check the conversions themselves). */
void gdsq_oracle_halves_to_floats(const uint16_t* h, float* f, uint64_t n) {
  for (uint64_t i = 0; i < n; ++i) f[i] = gdsq_oracle_half_to_float(h[i]);
}

void gdsq_oracle_floats_to_halves(const float* f, uint16_t* h, uint64_t n) {
  for (uint64_t i = 0; i < n; ++i) h[i] = gdsq_oracle_float_to_half(f[i]);
}

int gdsq_oracle_num_threads(void) {
#ifdef _OPENMP
  extern int omp_get_max_threads(void);
  return omp_get_max_threads();
#else
  return 1;
#endif
}
