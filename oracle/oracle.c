/*
 * CPU oracle for the gfxinfer-b200 decode path. TEST INFRASTRUCTURE ONLY:
 * tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg are its
 * only users. See oracle.h for the contract.
 *
 * Build flags matter: -ffp-contract=off (no silent a*b+c fusion) and no
 * -ffast-math, so every float operation below is one IEEE operation with
 * round-to-nearest-even, exactly as the CUDA kernels (built with -fmad=false)
 * perform them.
 */
#include "oracle.h"

#include <float.h>
#include <limits.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#ifdef _OPENMP
#include <omp.h>
#endif

#define GROUP 128u

/* ======================================================================== */
/* scalar helpers                                                           */
/* ======================================================================== */

static inline uint32_t f32_bits(float value) {
  uint32_t bits;
  memcpy(&bits, &value, sizeof bits);
  return bits;
}

static inline float bits_f32(uint32_t bits) {
  float value;
  memcpy(&value, &bits, sizeof value);
  return value;
}

/* IEEE binary32 -> binary16, round to nearest even (the rounding of
 * __float2half, used at every fp16 store in lowbit_gemv.hip / qwen_ops.hip). */
uint16_t or_f32_to_f16(float value) {
  const uint32_t x = f32_bits(value);
  const uint32_t sign = (x >> 16) & 0x8000u;
  const uint32_t magnitude = x & 0x7fffffffu;
  if (magnitude >= 0x7f800000u) {
    return (uint16_t)(sign | (magnitude > 0x7f800000u ? 0x7e00u : 0x7c00u));
  }
  if (magnitude >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);
  if (magnitude < 0x38800000u) {
    if (magnitude < 0x33000000u) return (uint16_t)sign;
    const uint32_t exponent = magnitude >> 23;
    const uint32_t mantissa = (magnitude & 0x7fffffu) | 0x800000u;
    const uint32_t shift = 126u - exponent;
    uint32_t quotient = mantissa >> shift;
    const uint32_t remainder = mantissa & ((1u << shift) - 1u);
    const uint32_t half = 1u << (shift - 1u);
    if (remainder > half || (remainder == half && (quotient & 1u))) ++quotient;
    return (uint16_t)(sign | quotient);
  }
  uint32_t rebased = magnitude - 0x38000000u;
  rebased += 0xfffu + ((rebased >> 13) & 1u);
  return (uint16_t)(sign | (rebased >> 13));
}

float or_f16_to_f32(uint16_t bits) {
  const uint32_t sign = ((uint32_t)bits & 0x8000u) << 16;
  uint32_t exponent = ((uint32_t)bits >> 10) & 0x1fu;
  uint32_t mantissa = (uint32_t)bits & 0x3ffu;
  if (exponent == 0) {
    if (mantissa == 0) return bits_f32(sign);
    /* subnormal half: normalise */
    int shift = 0;
    while ((mantissa & 0x400u) == 0) {
      mantissa <<= 1;
      ++shift;
    }
    mantissa &= 0x3ffu;
    return bits_f32(sign | ((uint32_t)(113 - shift) << 23) | (mantissa << 13));
  }
  if (exponent == 0x1f) return bits_f32(sign | 0x7f800000u | (mantissa << 13));
  return bits_f32(sign | ((exponent + 112u) << 23) | (mantissa << 13));
}

uint16_t or_f32_to_bf16(float value) {
  uint32_t x = f32_bits(value);
  if ((x & 0x7fffffffu) > 0x7f800000u) return 0x7fc0u;
  x += 0x7fffu + ((x >> 16) & 1u);
  return (uint16_t)(x >> 16);
}

/* qwen_ops.hip:27-29 */
float or_bf16_to_f32(uint16_t bits) { return bits_f32((uint32_t)bits << 16); }

static inline float pow2i(int k) { return bits_f32((uint32_t)(k + 127) << 23); }

/* e^x: Cody-Waite two-constant reduction x = n*ln2 + r (W. J. Cody and W. Waite,
 * "Software Manual for the Elementary Functions", 1980), e^r by its degree-7
 * Taylor polynomial in Horner form, then exact scaling by 2^n. */
float or_expf(float x) {
  if (x != x) return x;
  if (x > 88.7228394f) return INFINITY;
  if (x < -104.0f) return 0.0f;
  const float n = rintf(x * 1.44269502f);
  float r = fmaf(n, -0.693145751953125f, x);
  r = fmaf(n, -1.428606765330187e-6f, r);
  float p = 1.98412698e-4f;
  p = fmaf(p, r, 1.38888889e-3f);
  p = fmaf(p, r, 8.33333333e-3f);
  p = fmaf(p, r, 4.16666667e-2f);
  p = fmaf(p, r, 1.66666667e-1f);
  p = fmaf(p, r, 0.5f);
  p = fmaf(p, r, 1.0f);
  p = fmaf(p, r, 1.0f);
  const int e = (int)n;
  if (e > 127) return (p * pow2i(127)) * pow2i(e - 127);
  if (e < -126) return (p * pow2i(e + 64)) * pow2i(-64);
  return p * pow2i(e);
}

/* ln(u) for finite u >= 1: u = m*2^e with m in [sqrt(1/2), sqrt(2)],
 * ln(m) = 2*atanh(s), s = (m-1)/(m+1), by its odd series to s^11. */
static float or_log_ge1(float u) {
  uint32_t bits = f32_bits(u);
  int e = (int)((bits >> 23) & 0xffu) - 127;
  float m = bits_f32((bits & 0x007fffffu) | 0x3f800000u);
  if (m > 1.41421356f) {
    m = m * 0.5f;
    e += 1;
  }
  const float s = (m - 1.0f) / (m + 1.0f);
  const float s2 = s * s;
  float p = 0.0909090909f;
  p = fmaf(p, s2, 0.111111111f);
  p = fmaf(p, s2, 0.142857143f);
  p = fmaf(p, s2, 0.2f);
  p = fmaf(p, s2, 0.333333333f);
  p = fmaf(p, s2, 1.0f);
  const float lm = (2.0f * s) * p;
  return fmaf((float)e, 0.693147181f, lm);
}

/* log(1+x) for x >= 0 (D. Goldberg, "What Every Computer Scientist Should Know
 * About Floating-Point Arithmetic", 1991, Theorem 4). */
float or_log1pf(float x) {
  if (x != x) return x;
  if (x == INFINITY) return x;
  const float u = 1.0f + x;
  if (u == 1.0f) return x;
  return or_log_ge1(u) * (x / (u - 1.0f));
}

/* __float2int_rn semantics: NaN -> 0, saturating, ties to even. */
static inline int or_f2i_rn(float x) {
  if (x != x) return 0;
  if (x >= 2147483648.0f) return INT_MAX;
  if (x < -2147483648.0f) return INT_MIN;
  return (int)rintf(x);
}

static inline int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

static inline uint64_t mix64(uint64_t z) {
  z += 0x9e3779b97f4a7c15ULL;
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
  return z ^ (z >> 31);
}

/* Counter-based generator for synthetic weights (splitmix64 finaliser). */
uint64_t or_hash(uint64_t seed, uint64_t stream, uint64_t index) {
  return mix64(mix64(seed ^ (stream * 0xd1b54a32d192ed03ULL)) + index);
}

/* ======================================================================== */
/* packing: restates src/quantization.cpp                                  */
/* ======================================================================== */

/* quantization.cpp:15-27 */
static int nearest_w2(float normalized) {
  static const int levels[4] = {-3, -1, 1, 3};
  int best = levels[0];
  float best_error = INFINITY;
  for (int i = 0; i < 4; ++i) {
    const float error = fabsf(normalized - (float)levels[i]);
    if (error < best_error) {
      best = levels[i];
      best_error = error;
    }
  }
  return best;
}

/* quantization.cpp:29-46 */
static uint8_t encode_value(float value, float scale, int format) {
  const float normalized = scale == 0.0f ? 0.0f : value / scale;
  switch (format) {
    case OR_W2: return (uint8_t)((nearest_w2(normalized) + 3) / 2);
    case OR_W3: return (uint8_t)(clampi((int)nearbyintf(normalized), -4, 3) + 4);
    case OR_W4: return (uint8_t)(clampi((int)nearbyintf(normalized), -8, 7) & 0x0f);
    default: return 0;
  }
}

/* quantization.cpp:48-56 */
int or_decode_value(uint8_t code, int format) {
  switch (format) {
    case OR_W2: return (int)code * 2 - 3;
    case OR_W3: return (int)code - 4;
    case OR_W4: return (code & 0x08u) ? (int)code - 16 : (int)code;
    default: return 0;
  }
}

/* quantization.cpp:58-65 */
static float divisor_for(int format) {
  switch (format) {
    case OR_W2: return 3.0f;
    case OR_W3: return 4.0f;
    case OR_W4: return 8.0f;
    default: return 1.0f;
  }
}

/* quantization.cpp:67-92: four least-squares refits with double accumulators. */
static float choose_scale(const float* values, float maximum, int format) {
  if (maximum == 0.0f) return 1.0f;
  float scale = maximum / divisor_for(format);
  for (int iteration = 0; iteration < 4; ++iteration) {
    double numerator = 0.0;
    double denominator = 0.0;
    for (unsigned i = 0; i < GROUP; ++i) {
      const int level = or_decode_value(encode_value(values[i], scale, format), format);
      numerator += (double)values[i] * level;
      denominator += (double)level * level;
    }
    if (denominator == 0.0) break;
    scale = (float)(numerator / denominator);
  }
  return scale > FLT_MIN ? scale : FLT_MIN;
}

/* quantization.cpp:94-124 */
static void store_code(uint8_t* row, size_t column, uint8_t code, int format) {
  switch (format) {
    case OR_W2:
      row[column / 4] |= (uint8_t)((code & 0x03u) << ((column & 3u) * 2u));
      break;
    case OR_W3: {
      const size_t group = column / GROUP, local = column % GROUP;
      const size_t byte = local / 8;
      const unsigned bit = (unsigned)(local & 7u);
      for (size_t plane = 0; plane < 3; ++plane) {
        row[group * 48 + plane * 16 + byte] |= (uint8_t)(((code >> plane) & 1u) << bit);
      }
      break;
    }
    case OR_W4:
      row[column / 2] |= (uint8_t)((code & 0x0fu) << ((column & 1u) * 4u));
      break;
    default: break;
  }
}

/* quantization.cpp:126-150 */
uint8_t or_load_code(const uint8_t* row, size_t column, int format) {
  switch (format) {
    case OR_W2: return (uint8_t)((row[column / 4] >> ((column & 3u) * 2u)) & 0x03u);
    case OR_W3: {
      const size_t group = column / GROUP, local = column % GROUP;
      const size_t byte = local / 8;
      const unsigned bit = (unsigned)(local & 7u);
      uint8_t code = 0;
      for (size_t plane = 0; plane < 3; ++plane) {
        code |= (uint8_t)(((row[group * 48 + plane * 16 + byte] >> bit) & 1u) << plane);
      }
      return code;
    }
    case OR_W4: return (uint8_t)((row[column / 2] >> ((column & 1u) * 4u)) & 0x0fu);
    default: return 0;
  }
}

/* quantization.cpp:154-161 */
size_t or_packed_row_bytes(int format, size_t columns) {
  switch (format) {
    case OR_W2: return (columns + 3) / 4;
    case OR_W3: return (columns * 3 + 7) / 8;
    case OR_W4: return (columns + 1) / 2;
    default: return 0;
  }
}

/* quantization.cpp:163-220. Returns 0 (ok), 1 (invalid_argument) or
 * 4 (unsupported), the reference ErrorCode values (status.h:11-20). */
int or_quantize_group128(const float* weights, size_t rows, size_t columns, int format,
                         uint8_t* codes, float* scales) {
  if (rows == 0 || columns == 0 || columns % GROUP != 0) return 1;
  if (format != OR_W2 && format != OR_W3 && format != OR_W4) return 4;
  const size_t row_bytes = or_packed_row_bytes(format, columns);
  const size_t groups = columns / GROUP;
  memset(codes, 0, rows * row_bytes);
  int non_finite = 0;
#pragma omp parallel for schedule(static) reduction(| : non_finite)
  for (long long r = 0; r < (long long)rows; ++r) {
    const float* source = weights + (size_t)r * columns;
    uint8_t* destination = codes + (size_t)r * row_bytes;
    for (size_t g = 0; g < groups; ++g) {
      float maximum = 0.0f;
      for (size_t i = 0; i < GROUP; ++i) {
        const float value = source[g * GROUP + i];
        if (!isfinite(value)) {
          non_finite = 1;
          continue;
        }
        const float magnitude = fabsf(value);
        maximum = maximum > magnitude ? maximum : magnitude;
      }
      const float scale = choose_scale(source + g * GROUP, maximum, format);
      scales[(size_t)r * groups + g] = scale;
      for (size_t i = 0; i < GROUP; ++i) {
        const size_t column = g * GROUP + i;
        store_code(destination, column, encode_value(source[column], scale, format), format);
      }
    }
  }
  return non_finite ? 1 : 0;
}

/* quantization.cpp:222-235 */
float or_dequantized_weight(const uint8_t* codes, const float* scales, size_t rows,
                            size_t columns, int format, size_t row, size_t column) {
  if (row >= rows || column >= columns || columns % GROUP != 0) return NAN;
  const size_t row_bytes = or_packed_row_bytes(format, columns);
  const uint8_t code = or_load_code(codes + row * row_bytes, column, format);
  return (float)or_decode_value(code, format) * scales[row * (columns / GROUP) + column / GROUP];
}

/* quantization.cpp:253-318 */
int or_tile_gfx12(const uint8_t* codes, const float* scales, size_t rows, size_t columns,
                  int format, uint8_t* tiled_codes, float* tiled_scales) {
  if (rows == 0 || columns == 0 || rows % 16 != 0 || columns % GROUP != 0 ||
      (format != OR_W2 && format != OR_W3 && format != OR_W4)) {
    return 1;
  }
  const size_t row_bytes = or_packed_row_bytes(format, columns);
  const size_t groups = columns / GROUP;
  const size_t fragment = format == OR_W2 ? 8 : (format == OR_W3 ? 12 : 16);
  memset(tiled_codes, 0, rows * row_bytes);
  size_t destination = 0;
  for (size_t tile = 0; tile < rows / 16; ++tile) {
    for (size_t g = 0; g < groups; ++g) {
      for (size_t k_tile = 0; k_tile < 4; ++k_tile) {
        for (size_t local_row = 0; local_row < 16; ++local_row) {
          const size_t row = tile * 16 + local_row;
          if (format == OR_W3) {
            for (size_t item = 0; item < 32; ++item) {
              const size_t column = g * GROUP + k_tile * 32 + item;
              const uint8_t code = or_load_code(codes + row * row_bytes, column, format);
              const size_t bit = item * 3;
              const size_t byte = bit / 8;
              const unsigned shift = (unsigned)(bit & 7u);
              tiled_codes[destination + byte] |= (uint8_t)(code << shift);
              if (shift > 5u) {
                tiled_codes[destination + byte + 1] |= (uint8_t)(code >> (8u - shift));
              }
            }
          } else {
            memcpy(tiled_codes + destination,
                   codes + row * row_bytes + g * fragment * 4 + k_tile * fragment, fragment);
          }
          destination += fragment;
        }
      }
      for (size_t local_row = 0; local_row < 16; ++local_row) {
        tiled_scales[(tile * groups + g) * 16 + local_row] =
            scales[(tile * 16 + local_row) * groups + g];
      }
    }
  }
  return 0;
}

void or_unpack_logical(const uint8_t* codes, size_t rows, size_t columns, int format,
                       int8_t* logical) {
  const size_t row_bytes = or_packed_row_bytes(format, columns);
#pragma omp parallel for schedule(static)
  for (long long r = 0; r < (long long)rows; ++r) {
    for (size_t c = 0; c < columns; ++c) {
      logical[(size_t)r * columns + c] = (int8_t)or_decode_value(
          or_load_code(codes + (size_t)r * row_bytes, c, format), format);
    }
  }
}

/* ======================================================================== */
/* activation quantizers: lowbit_gemv.hip:373-436                           */
/* ======================================================================== */

static void quantize_group(const uint16_t* input, float divisor_value, int limit,
                           int* codes, uint16_t* scale_out) {
  float maximum = 0.0f;
  for (unsigned i = 0; i < GROUP; ++i) {
    const float magnitude = fabsf(or_f16_to_f32(input[i]));
    maximum = fmaxf(maximum, magnitude);
  }
  const uint16_t scale_bits =
      or_f32_to_f16(maximum == 0.0f ? 1.0f : maximum / divisor_value);
  *scale_out = scale_bits;
  const float scale = or_f16_to_f32(scale_bits);
  for (unsigned i = 0; i < GROUP; ++i) {
    codes[i] = clampi(or_f2i_rn(or_f16_to_f32(input[i]) / scale), -limit, limit);
  }
}

void or_quantize_activation_i4(const uint16_t* input, size_t columns, unsigned batch,
                               uint8_t* packed, uint16_t* scales) {
  const size_t groups = columns / GROUP;
  int codes[GROUP];
  for (unsigned b = 0; b < batch; ++b) {
    for (size_t g = 0; g < groups; ++g) {
      quantize_group(input + b * columns + g * GROUP, 7.0f, 7, codes, &scales[b * groups + g]);
      for (unsigned i = 0; i < GROUP / 2; ++i) {
        packed[b * (columns / 2) + g * 64 + i] =
            (uint8_t)((codes[2 * i] & 0x0f) | ((codes[2 * i + 1] & 0x0f) << 4));
      }
    }
  }
}

void or_quantize_activation_i8(const uint16_t* input, size_t columns, unsigned batch,
                               int8_t* quantized, uint16_t* scales) {
  const size_t groups = columns / GROUP;
  int codes[GROUP];
  for (unsigned b = 0; b < batch; ++b) {
    for (size_t g = 0; g < groups; ++g) {
      quantize_group(input + b * columns + g * GROUP, 127.0f, 127, codes,
                     &scales[b * groups + g]);
      for (unsigned i = 0; i < GROUP; ++i) quantized[b * columns + g * GROUP + i] = (int8_t)codes[i];
    }
  }
}

void or_unpack_a4(const uint8_t* packed, size_t count, int8_t* values) {
  for (size_t i = 0; i < count; ++i) {
    const uint8_t byte = packed[i / 2];
    int nibble = (i & 1u) ? (byte >> 4) : (byte & 0x0f);
    values[i] = (int8_t)(nibble >= 8 ? nibble - 16 : nibble);
  }
}

/* ======================================================================== */
/* GEMV: integer per-group dot, fp32 fma across groups in ascending order   */
/* (lowbit_gemv.hip:490-537 and 703-747).                                   */
/* ======================================================================== */

void or_gemv_int(const int8_t* weights, const uint16_t* weight_scales, size_t rows,
                 size_t columns, const int8_t* activations, const uint16_t* activation_scales,
                 unsigned batch, float* output) {
  const size_t groups = columns / GROUP;
#pragma omp parallel for schedule(static)
  for (long long r = 0; r < (long long)rows; ++r) {
    const int8_t* w = weights + (size_t)r * columns;
    for (unsigned b = 0; b < batch; ++b) {
      const int8_t* a = activations + (size_t)b * columns;
      float accumulator = 0.0f;
      for (size_t g = 0; g < groups; ++g) {
        int dot = 0;
        for (unsigned i = 0; i < GROUP; ++i) dot += (int)w[g * GROUP + i] * (int)a[g * GROUP + i];
        const float product = or_f16_to_f32(weight_scales[(size_t)r * groups + g]) *
                              or_f16_to_f32(activation_scales[(size_t)b * groups + g]);
        accumulator = fmaf((float)dot, product, accumulator);
      }
      output[(size_t)b * rows + (size_t)r] = accumulator;
    }
  }
}

/* FP16-activation path (lowbit_gemv.hip:757-834): weight = fp16(q * scale),
 * products accumulated exactly in double; used as a tolerance reference. */
void or_gemv_f16(const int8_t* weights, const uint16_t* weight_scales, size_t rows,
                 size_t columns, const uint16_t* activations, unsigned batch, double* output) {
  const size_t groups = columns / GROUP;
#pragma omp parallel for schedule(static)
  for (long long r = 0; r < (long long)rows; ++r) {
    for (unsigned b = 0; b < batch; ++b) {
      double sum = 0.0;
      for (size_t c = 0; c < columns; ++c) {
        const float scale = or_f16_to_f32(weight_scales[(size_t)r * groups + c / GROUP]);
        const float w = or_f16_to_f32(or_f32_to_f16((float)weights[(size_t)r * columns + c] * scale));
        sum += (double)w * (double)or_f16_to_f32(activations[(size_t)b * columns + c]);
      }
      output[(size_t)b * rows + (size_t)r] = sum;
    }
  }
}

/* ======================================================================== */
/* qwen ops                                                                 */
/* ======================================================================== */

/* Pairwise tree of a 32-lane warp reduction (lane 0's result of the
 * shuffle-down sequence 16, 8, 4, 2, 1; qwen_ops.hip:18-25). */
float or_tree32(const float* values) {
  float a[32];
  memcpy(a, values, sizeof a);
  for (unsigned offset = 16; offset != 0; offset >>= 1) {
    for (unsigned i = 0; i < offset; ++i) a[i] = a[i] + a[i + offset];
  }
  return a[0];
}

/* Block of 256 threads, thread t accumulating elements t, t+256, ... with fma,
 * then the warp tree and the tree over the eight warp sums (qwen_ops.hip:38-55). */
static float block256_square_sum(const float* values, size_t elements) {
  float partial[256];
  for (unsigned t = 0; t < 256; ++t) {
    float sum = 0.0f;
    for (size_t i = t; i < elements; i += 256) sum = fmaf(values[i], values[i], sum);
    partial[t] = sum;
  }
  float waves[32] = {0};
  for (unsigned w = 0; w < 8; ++w) waves[w] = or_tree32(partial + 32 * w);
  return or_tree32(waves);
}

static float inverse_rms(float square_sum, size_t elements, float eps) {
  const float mean = square_sum / (float)elements;
  return 1.0f / sqrtf(mean + eps);
}

/* qwen_ops.hip:31-63 */
void or_rms_norm(const uint16_t* input, const uint16_t* weight, size_t elements, float eps,
                 int unit_offset, uint16_t* output) {
  float* values = (float*)malloc(elements * sizeof(float));
  for (size_t i = 0; i < elements; ++i) values[i] = or_f16_to_f32(input[i]);
  const float inv = inverse_rms(block256_square_sum(values, elements), elements, eps);
  for (size_t i = 0; i < elements; ++i) {
    float scale = or_bf16_to_f32(weight[i]);
    if (unit_offset) scale += 1.0f;
    output[i] = or_f32_to_f16((values[i] * inv) * scale);
  }
  free(values);
}

/* qwen_ops.hip:176-217 */
void or_residual_add_rms_norm(const uint16_t* residual, const float* update,
                              const uint16_t* weight, size_t elements, float eps,
                              int unit_offset, uint16_t* residual_out, uint16_t* normalized) {
  float* values = (float*)malloc(elements * sizeof(float));
  for (size_t i = 0; i < elements; ++i) {
    const uint16_t rounded = or_f32_to_f16(or_f16_to_f32(residual[i]) + update[i]);
    residual_out[i] = rounded;
    values[i] = or_f16_to_f32(rounded);
  }
  const float inv = inverse_rms(block256_square_sum(values, elements), elements, eps);
  for (size_t i = 0; i < elements; ++i) {
    float scale = or_bf16_to_f32(weight[i]);
    if (unit_offset) scale += 1.0f;
    normalized[i] = or_f32_to_f16((values[i] * inv) * scale);
  }
  free(values);
}

/* qwen_ops.hip:108-118 and 134-136 */
void or_silu_multiply_f16(const float* gate, const float* up, size_t elements,
                          uint16_t* output) {
  for (size_t i = 0; i < elements; ++i) {
    const float g = gate[i];
    output[i] = or_f32_to_f16((g / (1.0f + or_expf(-g))) * up[i]);
  }
}

/* qwen_ops.hip:219-261 */
void or_gdn_conv_update(const float* projected, const uint16_t* weight, uint16_t* state,
                        uint16_t* output, uint16_t* appended_log, size_t channels,
                        unsigned batch) {
#pragma omp parallel for schedule(static)
  for (long long cc = 0; cc < (long long)channels; ++cc) {
    const size_t c = (size_t)cc;
    uint16_t taps[4];
    memcpy(taps, state + c * 4, sizeof taps);
    for (unsigned t = 0; t < batch; ++t) {
      taps[0] = taps[1];
      taps[1] = taps[2];
      taps[2] = taps[3];
      taps[3] = or_f32_to_f16(projected[(size_t)t * channels + c]);
      if (appended_log) appended_log[(size_t)t * channels + c] = taps[3];
      float conv = 0.0f;
      for (unsigned k = 0; k < 4; ++k) {
        conv = fmaf(or_f16_to_f32(taps[k]), or_bf16_to_f32(weight[c * 4 + k]), conv);
      }
      output[(size_t)t * channels + c] = or_f32_to_f16(conv / (1.0f + or_expf(-conv)));
    }
    memcpy(state + c * 4, taps, sizeof taps);
  }
}

/* Sum of 128 per-thread values held by warps 0..3 of a 256-thread block
 * (warps 4..7 contribute zero): qwen_ops.hip:314-332, 393-399. */
static float block128_sum(const float* values) {
  float waves[32] = {0};
  for (unsigned w = 0; w < 4; ++w) waves[w] = or_tree32(values + 32 * w);
  return or_tree32(waves);
}

/* qwen_ops.hip:263-411. State layout S[value_head][k][v]. */
void or_gdn_recurrent(const uint16_t* qkv, const float* z, const float* a, const float* b,
                      const uint16_t* a_log, const uint16_t* dt_bias,
                      const uint16_t* norm_weight, float* state, uint16_t* output,
                      float* key_log, float* delta_log, float* decay_log, unsigned key_heads,
                      unsigned value_heads, unsigned batch) {
  const unsigned head = 128;
  const unsigned key_elements = key_heads * head;
  const unsigned value_elements = value_heads * head;
  const unsigned channels = 2 * key_elements + value_elements;
  const unsigned ratio = value_heads / key_heads;
#pragma omp parallel for schedule(static)
  for (int vhh = 0; vhh < (int)value_heads; ++vhh) {
    const unsigned vh = (unsigned)vhh;
    const unsigned kh = vh / ratio;
    float* S = state + (size_t)vh * head * head;
    for (unsigned t = 0; t < batch; ++t) {
      const uint16_t* token_qkv = qkv + (size_t)t * channels;
      float q[128], k[128], sq[128], sk[128];
      for (unsigned i = 0; i < head; ++i) {
        q[i] = or_f16_to_f32(token_qkv[kh * head + i]);
        k[i] = or_f16_to_f32(token_qkv[key_elements + kh * head + i]);
        sq[i] = q[i] * q[i];
        sk[i] = k[i] * k[i];
      }
      const float inv_q = (1.0f / sqrtf(block128_sum(sq) + 1.0e-6f)) * 0.08838834764831845f;
      const float inv_k = 1.0f / sqrtf(block128_sum(sk) + 1.0e-6f);
      const float a_value = a[(size_t)t * value_heads + vh] + or_bf16_to_f32(dt_bias[vh]);
      const float softplus = a_value > 20.0f ? a_value : or_log1pf(or_expf(a_value));
      const float g = -or_expf(or_bf16_to_f32(a_log[vh])) * softplus;
      const float decay = or_expf(g);
      const float beta = 1.0f / (1.0f + or_expf(-b[(size_t)t * value_heads + vh]));
      for (unsigned i = 0; i < head; ++i) {
        q[i] = q[i] * inv_q;
        k[i] = k[i] * inv_k;
      }
      if (decay_log) decay_log[(size_t)t * value_heads + vh] = decay;
      if (key_log && vh % ratio == 0) {
        for (unsigned i = 0; i < head; ++i) key_log[(size_t)t * key_elements + kh * head + i] = k[i];
      }
      float out[128], out_sq[128];
      for (unsigned v = 0; v < head; ++v) {
        float column[128];
        float memory = 0.0f;
        for (unsigned kk = 0; kk < head; ++kk) {
          column[kk] = S[kk * head + v] * decay;
          memory = fmaf(column[kk], k[kk], memory);
        }
        const float value = or_f16_to_f32(token_qkv[2 * key_elements + vh * head + v]);
        const float delta = (value - memory) * beta;
        if (delta_log) delta_log[(size_t)t * value_elements + vh * head + v] = delta;
        float mixed = 0.0f;
        for (unsigned kk = 0; kk < head; ++kk) {
          const float updated = fmaf(k[kk], delta, column[kk]);
          S[kk * head + v] = updated;
          mixed = fmaf(updated, q[kk], mixed);
        }
        out[v] = mixed;
        out_sq[v] = mixed * mixed;
      }
      const float inv_o = 1.0f / sqrtf(block128_sum(out_sq) / 128.0f + 1.0e-6f);
      for (unsigned v = 0; v < head; ++v) {
        const float zv = z[(size_t)t * value_elements + vh * head + v];
        const float gate = zv / (1.0f + or_expf(-zv));
        const float normalized = (out[v] * inv_o) * or_bf16_to_f32(norm_weight[v]);
        output[(size_t)t * value_elements + vh * head + v] = or_f32_to_f16(normalized * gate);
      }
    }
  }
}

/* qwen_ops.hip:413-539: replay the accepted prefix of the logs. */
void or_gdn_restore(uint16_t* conv_state, float* state, const uint16_t* conv_log,
                    const float* key_log, const float* delta_log, const float* decay_log,
                    size_t channels, unsigned key_heads, unsigned value_heads,
                    unsigned accepted) {
  for (size_t c = 0; c < channels; ++c) {
    uint16_t* taps = conv_state + c * 4;
    for (unsigned t = 0; t < accepted; ++t) {
      taps[0] = taps[1];
      taps[1] = taps[2];
      taps[2] = taps[3];
      taps[3] = conv_log[(size_t)t * channels + c];
    }
  }
  const unsigned head = 128, ratio = value_heads / key_heads;
  for (unsigned vh = 0; vh < value_heads; ++vh) {
    float* S = state + (size_t)vh * head * head;
    const unsigned kh = vh / ratio;
    for (unsigned t = 0; t < accepted; ++t) {
      const float decay = decay_log[(size_t)t * value_heads + vh];
      for (unsigned kk = 0; kk < head; ++kk) {
        const float key = key_log[(size_t)t * key_heads * head + kh * head + kk];
        for (unsigned v = 0; v < head; ++v) {
          const float delta = delta_log[(size_t)t * value_heads * head + vh * head + v];
          S[kk * head + v] = fmaf(key, delta, S[kk * head + v] * decay);
        }
      }
    }
  }
}

/* RoPE angle table: inv_freq = theta^(-2f/rotary), angle = fp32(position*inv_freq)
 * (qwen_ops.hip:662-672), cos/sin evaluated in double and rounded once. */
void or_rope_table(size_t positions, unsigned rotary, float theta, float* cos_table,
                   float* sin_table) {
  const unsigned half = rotary / 2;
  for (size_t p = 0; p < positions; ++p) {
    for (unsigned f = 0; f < half; ++f) {
      const float exponent = (2.0f * (float)f) / (float)rotary;
      const float inv_freq = (float)pow((double)theta, -(double)exponent);
      const float angle = (float)p * inv_freq;
      cos_table[p * half + f] = (float)cos((double)angle);
      sin_table[p * half + f] = (float)sin((double)angle);
    }
  }
}

/* qwen_ops.hip:599-676, head size 256. */
void or_qk_norm_rope(const float* input, size_t stride, const uint16_t* weight,
                     unsigned heads, size_t position, const float* cos_table,
                     const float* sin_table, unsigned rotary, uint16_t* output) {
  const unsigned head = 256, half = rotary / 2;
  for (unsigned h = 0; h < heads; ++h) {
    float v[256], sq[256], n[256];
    for (unsigned d = 0; d < head; ++d) {
      v[d] = input[h * stride + d];
      sq[d] = v[d] * v[d];
    }
    float waves[32] = {0};
    for (unsigned w = 0; w < 8; ++w) waves[w] = or_tree32(sq + 32 * w);
    const float inv = 1.0f / sqrtf(or_tree32(waves) / 256.0f + 1.0e-6f);
    for (unsigned d = 0; d < head; ++d) n[d] = v[d] * (inv * (1.0f + or_bf16_to_f32(weight[d])));
    for (unsigned d = 0; d < head; ++d) {
      float value = n[d];
      if (d < rotary) {
        const unsigned f = d % half;
        const float partner = d < half ? n[d + half] : n[d - half];
        const float rotated = d < half ? -partner : partner;
        value = fmaf(value, cos_table[position * half + f], rotated * sin_table[position * half + f]);
      }
      output[h * head + d] = or_f32_to_f16(value);
    }
  }
}

#define OR_ATTN_CHUNK 128u

/* qwen_ops.hip:698-766 restated as chunked online softmax: positions are split
 * into chunks of 128; each chunk runs the reference's serial online update;
 * chunks are merged in ascending order. Scores: lane l of a warp owns dims
 * 8l..8l+7 (fma chain), then the 32-lane tree; scale 1/16. */
void or_gated_attention(const uint16_t* query, const float* gate_projection,
                        const uint16_t* key_cache, const uint16_t* value_cache,
                        size_t token_count, unsigned q_heads, unsigned kv_heads,
                        uint16_t* output) {
  const unsigned head = 256;
  const unsigned group = q_heads / kv_heads;
  const size_t chunks = (token_count + OR_ATTN_CHUNK - 1) / OR_ATTN_CHUNK;
#pragma omp parallel for schedule(static)
  for (int hh = 0; hh < (int)q_heads; ++hh) {
    const unsigned h = (unsigned)hh;
    const unsigned kvh = h / group;
    float q[256];
    for (unsigned d = 0; d < head; ++d) q[d] = or_f16_to_f32(query[h * head + d]);
    float M = -INFINITY, Den = 0.0f, Acc[256];
    for (size_t c = 0; c < chunks; ++c) {
      float m = -INFINITY, den = 0.0f, acc[256];
      for (unsigned d = 0; d < head; ++d) acc[d] = 0.0f;
      const size_t end = (c + 1) * OR_ATTN_CHUNK < token_count ? (c + 1) * OR_ATTN_CHUNK : token_count;
      for (size_t p = c * OR_ATTN_CHUNK; p < end; ++p) {
        const uint16_t* key = key_cache + (p * kv_heads + kvh) * head;
        const uint16_t* value = value_cache + (p * kv_heads + kvh) * head;
        float lanes[32];
        for (unsigned l = 0; l < 32; ++l) {
          float s = 0.0f;
          for (unsigned j = 0; j < 8; ++j) s = fmaf(q[8 * l + j], or_f16_to_f32(key[8 * l + j]), s);
          lanes[l] = s;
        }
        const float score = or_tree32(lanes) * 0.0625f;
        const float next = fmaxf(m, score);
        const float alpha = or_expf(m - next);
        const float beta = or_expf(score - next);
        den = den * alpha + beta;
        for (unsigned d = 0; d < head; ++d) acc[d] = acc[d] * alpha + or_f16_to_f32(value[d]) * beta;
        m = next;
      }
      if (c == 0) {
        M = m;
        Den = den;
        memcpy(Acc, acc, sizeof Acc);
      } else {
        const float next = fmaxf(M, m);
        const float a1 = or_expf(M - next);
        const float a2 = or_expf(m - next);
        Den = Den * a1 + den * a2;
        for (unsigned d = 0; d < head; ++d) Acc[d] = Acc[d] * a1 + acc[d] * a2;
        M = next;
      }
    }
    for (unsigned d = 0; d < head; ++d) {
      const float gate = gate_projection[h * head * 2 + head + d];
      const float gate_scale = 1.0f / (1.0f + or_expf(-gate));
      output[h * head + d] = or_f32_to_f16((Acc[d] / Den) * gate_scale);
    }
  }
}

/* qwen_ops.hip:768-807: first maximum, lowest index on ties. */
uint32_t or_argmax(const float* logits, size_t count) {
  float best = -INFINITY;
  uint32_t index = 0;
  for (size_t i = 0; i < count; ++i) {
    if (logits[i] > best) {
      best = logits[i];
      index = (uint32_t)i;
    }
  }
  return index;
}

/* ======================================================================== */
/* synthetic weights                                                        */
/* ======================================================================== */

enum {
  K_INPUT_NORM = 0, K_POST_NORM, K_GATE, K_UP, K_DOWN,
  K_QKV, K_Z, K_A, K_B, K_CONV, K_ALOG, K_DTBIAS, K_GDN_NORM, K_GDN_OUT,
  K_Q, K_K, K_V, K_QNORM, K_KNORM, K_O,
  K_FC, K_PRE_EMB_NORM, K_PRE_HIDDEN_NORM, K_MTP_FINAL_NORM
};
#define LAYER_GLOBAL 4096u
#define LAYER_MTP 4097u
enum { G_EMBEDDING = 0, G_FINAL_NORM = 1, G_LM_HEAD = 2 };

static uint32_t tensor_id(uint32_t layer, uint32_t kind) { return layer * 32u + kind; }

static int format_of_bits(uint32_t bits) {
  return bits == 2 ? OR_W2 : (bits == 3 ? OR_W3 : OR_W4);
}

static void scale_range(int format, float* lo, float* hi) {
  switch (format) {
    case OR_W2: *lo = 0.0045f; *hi = 0.0134f; break;
    case OR_W3: *lo = 0.0050f; *hi = 0.0150f; break;
    default: *lo = 0.0023f; *hi = 0.0069f; break;
  }
}

static inline float unit_float(uint64_t h) {
  return (float)(h >> 40) * (1.0f / 16777216.0f);
}

/* Zero-mean synthetic codes: W2 levels {-3,-1,1,3} (top two hash bits), W3 q
 * uniform on {-3..3}, W4 q uniform on {-7..7}; returned as reference codes. */
static inline uint8_t synthetic_code(uint64_t seed, uint32_t tensor, size_t index, int format) {
  const uint64_t h = or_hash(seed, 2ull * tensor, index);
  if (format == OR_W2) return (uint8_t)(h >> 62);
  if (format == OR_W3) return (uint8_t)((h >> 32) % 7u + 1u);
  return (uint8_t)(((int)((h >> 32) % 15u) - 7) & 0x0f);
}

void or_gen_codes_rowmajor(uint64_t seed, uint32_t tensor, size_t rows, size_t columns,
                           int format, uint8_t* codes) {
  const size_t row_bytes = or_packed_row_bytes(format, columns);
  memset(codes, 0, rows * row_bytes);
#pragma omp parallel for schedule(static)
  for (long long r = 0; r < (long long)rows; ++r) {
    for (size_t c = 0; c < columns; ++c) {
      store_code(codes + (size_t)r * row_bytes, c,
                 synthetic_code(seed, tensor, (size_t)r * columns + c, format), format);
    }
  }
}

void or_gen_scales(uint64_t seed, uint32_t tensor, size_t count, int format,
                   uint16_t* scales) {
  float lo, hi;
  scale_range(format, &lo, &hi);
  for (size_t i = 0; i < count; ++i) {
    scales[i] = or_f32_to_f16(fmaf(hi - lo, unit_float(or_hash(seed, 2ull * tensor + 1, i)), lo));
  }
}

void or_gen_bf16(uint64_t seed, uint32_t tensor, size_t count, float lo, float hi,
                 uint16_t* values) {
  for (size_t i = 0; i < count; ++i) {
    values[i] = or_f32_to_bf16(fmaf(hi - lo, unit_float(or_hash(seed, 2ull * tensor, i)), lo));
  }
}

uint32_t or_prompt_token(uint64_t seed, uint32_t vocab, uint32_t index) {
  return (uint32_t)(or_hash(seed, 0xffffffull, index) % vocab);
}

/* ======================================================================== */
/* scalar forward (qwen_runtime.cpp:349-419, 715-867, 1264-1392)            */
/*                                                                          */
/* Tokens run in layer-major blocks of up to OR_BLOCK tokens, the order of  */
/* the reference's causal block_step: every projection of a layer is       */
/* applied to all of the block's tokens with one pass over the weights, the */
/* recurrent and attention steps then run token by token. The arithmetic of */
/* each token is the serial greedy step's, so a block gives the same bits   */
/* as the same tokens stepped one at a time.                                */
/* ======================================================================== */

#define OR_BLOCK 64u

/* A quantized matrix held packed so that the full-size models fit in host
 * memory: 2 bits per code for W2 (the reference code c, q = 2c - 3) and a
 * two's-complement nibble q for W3 and W4. Within each 128-column group,
 * byte j holds columns (8/bits)*j + k at bit k*bits, k = 0 .. 8/bits - 1, so
 * that the GEMV dots each bit plane against the matching activation plane. */
typedef struct {
  size_t rows, columns;
  unsigned bits;      /* storage bits per code: 2 or 4 */
  uint8_t* packed;    /* [rows][columns * bits / 8] */
  uint16_t* scales;   /* fp16 [rows][columns/128] */
} or_matrix;

static inline int matrix_code(const or_matrix* m, size_t row, size_t column) {
  const unsigned per_byte = 8u / m->bits, group_bytes = GROUP / per_byte;
  const size_t g = column / GROUP, c = column % GROUP;
  const uint8_t byte = m->packed[row * (m->columns / per_byte) + g * group_bytes + c / per_byte];
  const unsigned k = (unsigned)(c % per_byte);
  if (m->bits == 2) return 2 * (int)((byte >> (2u * k)) & 3u) - 3;
  return k == 0 ? (int)(int8_t)(uint8_t)(byte << 4) >> 4 : (int)(int8_t)byte >> 4;
}

typedef struct {
  int attention;
  unsigned state_index;
  uint16_t *input_norm, *post_norm;
  or_matrix gate, up, down;
  or_matrix qkv, z, a, b, out;
  uint16_t *conv, *a_log, *dt_bias, *gdn_norm;
  or_matrix q, k, v;
  uint16_t *q_norm, *k_norm;
} or_layer;

struct or_model {
  or_model_config cfg;
  int has_mtp;
  unsigned resident_layers; /* layers with their own weights; layer i uses those of i % resident_layers */
  or_layer* layers;
  or_layer mtp;
  or_matrix embedding, lm_head, fc;
  uint16_t *final_norm, *pre_emb_norm, *pre_hidden_norm, *mtp_final_norm;
  /* state */
  uint16_t* conv_states;
  float* gdn_states;
  uint16_t *key_caches, *value_caches, *mtp_keys, *mtp_values;
  float *rope_cos, *rope_sin;
  size_t position, mtp_position;
  int mtp_chain_active;
  /* activations, [OR_BLOCK][width] each */
  uint16_t *hidden, *next_hidden, *normalized, *post_attention, *post_normalized;
  uint16_t *conv_out, *mixer_out, *query, *key, *attn_out, *activated, *last_hidden, *mtp_hidden;
  uint16_t *mtp_concat, *mtp_input;
  float *proj_main, *proj_z, *proj_a, *proj_b, *proj_k, *proj_v, *update, *gate, *up, *logits;
  const float* last_logits;
  int8_t* act_planes;    /* [OR_BLOCK][widest]: codes in bit-plane order */
  int32_t* act_sums;     /* [OR_BLOCK][widest/128]: code sum per group */
  uint16_t* act_scales;  /* [OR_BLOCK][widest/128] */
  float* act_scale_values; /* [OR_BLOCK][widest/128]: the fp16 scales as floats */
  int8_t* act_codes;     /* [OR_BLOCK][widest] codes in column order */
  uint8_t* act_packed;   /* [OR_BLOCK][widest/2] */
  size_t widest;
  double layer_seconds, head_seconds;
  size_t tokens;
};

static void matrix_create(or_matrix* m, uint64_t seed, uint32_t tensor, size_t rows,
                          size_t columns, uint32_t bits) {
  const int format = format_of_bits(bits);
  m->rows = rows;
  m->columns = columns;
  m->bits = format == OR_W2 ? 2u : 4u;
  const unsigned per_byte = 8u / m->bits, group_bytes = GROUP / per_byte;
  const size_t row_bytes = columns / per_byte;
  m->packed = (uint8_t*)calloc(rows * row_bytes, 1);
  m->scales = (uint16_t*)malloc(rows * (columns / GROUP) * sizeof(uint16_t));
#pragma omp parallel for schedule(static)
  for (long long r = 0; r < (long long)rows; ++r) {
    uint8_t* row = m->packed + (size_t)r * row_bytes;
    for (size_t c = 0; c < columns; ++c) {
      const size_t index = (size_t)r * columns + c;
      const uint8_t code = synthetic_code(seed, tensor, index, format);
      const int q = or_decode_value(code, format);
      const size_t g = c / GROUP, within = c % GROUP;
      const unsigned k = (unsigned)(within % per_byte);
      const uint8_t stored = format == OR_W2 ? code : (uint8_t)(q & 15);
      row[g * group_bytes + within / per_byte] |= (uint8_t)(stored << (k * m->bits));
    }
  }
  or_gen_scales(seed, tensor, rows * (columns / GROUP), format, m->scales);
}

static void matrix_free(or_matrix* m) {
  free(m->packed);
  free(m->scales);
}

/* Integer dot of one packed 128-group with one token's activation planes:
 * sum over the group of q * a, exact in int32. Nibbles: q = (n ^ 8) - 8 with
 * n ^ 8 in [0, 15]; W2: q = 2c - 3 with c in [0, 3]. The unsigned part runs
 * on 8-bit multiply-adds (16-bit pair sums stay below 2^15) and the offset
 * comes from the group's activation sum. */
#if defined(__AVX2__)
#include <immintrin.h>
static inline int hsum_epi32(__m256i v) {
  __m128i x = _mm_add_epi32(_mm256_castsi256_si128(v), _mm256_extracti128_si256(v, 1));
  x = _mm_add_epi32(x, _mm_shuffle_epi32(x, 0x4e));
  x = _mm_add_epi32(x, _mm_shuffle_epi32(x, 0xb1));
  return _mm_cvtsi128_si32(x);
}
/* The unsigned parts of one packed group, four 32-byte planes. */
typedef struct {
  __m256i u[4];
} group_planes;
static inline group_planes unpack4(const uint8_t* w) {
  const __m256i low = _mm256_set1_epi8(0x0f), eight = _mm256_set1_epi8(0x08);
  const __m256i b0 = _mm256_loadu_si256((const __m256i*)w);
  const __m256i b1 = _mm256_loadu_si256((const __m256i*)(w + 32));
  group_planes g;
  g.u[0] = _mm256_xor_si256(_mm256_and_si256(b0, low), eight);
  g.u[1] = _mm256_xor_si256(_mm256_and_si256(b1, low), eight);
  g.u[2] = _mm256_xor_si256(_mm256_and_si256(_mm256_srli_epi16(b0, 4), low), eight);
  g.u[3] = _mm256_xor_si256(_mm256_and_si256(_mm256_srli_epi16(b1, 4), low), eight);
  return g;
}
static inline group_planes unpack2(const uint8_t* w) {
  const __m256i three = _mm256_set1_epi8(0x03);
  const __m256i b = _mm256_loadu_si256((const __m256i*)w);
  group_planes g;
  g.u[0] = _mm256_and_si256(b, three);
  g.u[1] = _mm256_and_si256(_mm256_srli_epi16(b, 2), three);
  g.u[2] = _mm256_and_si256(_mm256_srli_epi16(b, 4), three);
  g.u[3] = _mm256_and_si256(_mm256_srli_epi16(b, 6), three);
  return g;
}
/* sum over the group of u * a (the unsigned weight parts times the activation planes) */
static inline int planes_dot(const group_planes* g, const int8_t* p) {
  __m256i d = _mm256_maddubs_epi16(g->u[0], _mm256_loadu_si256((const __m256i*)p));
  d = _mm256_add_epi16(d, _mm256_maddubs_epi16(g->u[1], _mm256_loadu_si256((const __m256i*)(p + 32))));
  d = _mm256_add_epi16(d, _mm256_maddubs_epi16(g->u[2], _mm256_loadu_si256((const __m256i*)(p + 64))));
  d = _mm256_add_epi16(d, _mm256_maddubs_epi16(g->u[3], _mm256_loadu_si256((const __m256i*)(p + 96))));
  return hsum_epi32(_mm256_madd_epi16(d, _mm256_set1_epi16(1)));
}
#define OR_SIMD 1
#endif

/* Quantizes `count` fp16 rows of width K (launch_matrix's activation step,
 * qwen_runtime.cpp:78-148) into the model's plane/sum/scale buffers. */
static void quantize_rows(or_model* m, const uint16_t* input, size_t K, unsigned count, unsigned bits_per_code) {
  const unsigned per_byte = 8u / bits_per_code, group_bytes = GROUP / per_byte;
  const size_t groups = K / GROUP;
#pragma omp parallel for schedule(static)
  for (int tt = 0; tt < (int)count; ++tt) {
    const unsigned t = (unsigned)tt;
    const uint16_t* x = input + (size_t)t * K;
    uint16_t* scales = m->act_scales + (size_t)t * (m->widest / GROUP);
    int8_t* codes = m->act_codes + (size_t)t * m->widest;
    if (m->cfg.activation_bits == 8) {
      or_quantize_activation_i8(x, K, 1, codes, scales);
    } else {
      uint8_t* packed = m->act_packed + (size_t)t * (m->widest / 2 + 1);
      or_quantize_activation_i4(x, K, 1, packed, scales);
      or_unpack_a4(packed, K, codes);
    }
    int8_t* planes = m->act_planes + (size_t)t * m->widest;
    int32_t* sums = m->act_sums + (size_t)t * (m->widest / GROUP);
    float* scale_values = m->act_scale_values + (size_t)t * (m->widest / GROUP);
    for (size_t g = 0; g < groups; ++g) {
      scale_values[g] = or_f16_to_f32(scales[g]);
      int sum = 0;
      for (unsigned k = 0; k < per_byte; ++k) {
        for (unsigned j = 0; j < group_bytes; ++j) {
          const int8_t a = codes[g * GROUP + per_byte * j + k];
          planes[g * GROUP + k * group_bytes + j] = a;
          sum += a;
        }
      }
      sums[g] = sum;
    }
  }
}

/* y[t][r] for the first `rows` rows and `count` tokens: per 128-group an exact
 * int32 dot, then fp32 fma(dot, ws * as, acc) over the groups in ascending
 * order (or_gemv_int's arithmetic, lowbit_gemv.hip:490-537). Quantizes the
 * input first. */
static void apply_block_rows(or_model* m, const or_matrix* w, size_t rows, const uint16_t* input,
                             unsigned count, float* output) {
  const size_t K = w->columns, groups = K / GROUP;
  quantize_rows(m, input, K, count, w->bits);
  const unsigned per_byte = 8u / w->bits, group_bytes = GROUP / per_byte;
  const size_t row_bytes = K / per_byte, stride = m->widest, scale_stride = m->widest / GROUP;
#pragma omp parallel for schedule(static)
  for (long long r = 0; r < (long long)rows; ++r) {
    const uint8_t* row = w->packed + (size_t)r * row_bytes;
    float accumulator[OR_BLOCK];
    for (unsigned t = 0; t < count; ++t) accumulator[t] = 0.0f;
    for (size_t g = 0; g < groups; ++g) {
      const uint8_t* b = row + g * group_bytes;
      const float ws = or_f16_to_f32(w->scales[(size_t)r * groups + g]);
#if defined(OR_SIMD)
      /* nibbles: q = (n ^ 8) - 8; W2: q = 2c - 3 (the unsigned parts run on 8-bit multiply-adds,
       * 16-bit pair sums stay below 2^15, the offset comes from the group's activation sum) */
      const group_planes planes = w->bits == 4 ? unpack4(b) : unpack2(b);
      for (unsigned t = 0; t < count; ++t) {
        const int8_t* p = m->act_planes + (size_t)t * stride + g * GROUP;
        const int sum = m->act_sums[(size_t)t * scale_stride + g];
        const int u = planes_dot(&planes, p);
        const int dot = w->bits == 4 ? u - 8 * sum : 2 * u - 3 * sum;
        const float product = ws * m->act_scale_values[(size_t)t * scale_stride + g];
        accumulator[t] = fmaf((float)dot, product, accumulator[t]);
      }
#else
      for (unsigned t = 0; t < count; ++t) {
        const int8_t* p = m->act_planes + (size_t)t * stride + g * GROUP;
        int dot = 0;
        if (w->bits == 4) {
          for (unsigned j = 0; j < 64; ++j) {
            dot += ((int)(int8_t)(uint8_t)(b[j] << 4) >> 4) * (int)p[j] + ((int)(int8_t)b[j] >> 4) * (int)p[64 + j];
          }
        } else {
          for (unsigned j = 0; j < 32; ++j) {
            for (unsigned k = 0; k < 4; ++k) dot += (2 * (int)((b[j] >> (2 * k)) & 3) - 3) * (int)p[32 * k + j];
          }
        }
        const float product = ws * m->act_scale_values[(size_t)t * scale_stride + g];
        accumulator[t] = fmaf((float)dot, product, accumulator[t]);
      }
#endif
    }
    for (unsigned t = 0; t < count; ++t) output[(size_t)t * rows + (size_t)r] = accumulator[t];
  }
}

static void apply_block(or_model* m, const or_matrix* w, const uint16_t* input, unsigned count,
                        float* output) {
  apply_block_rows(m, w, w->rows, input, count, output);
}

static uint16_t* bf16_create(uint64_t seed, uint32_t tensor, size_t count, float lo, float hi) {
  uint16_t* values = (uint16_t*)malloc(count * sizeof(uint16_t));
  or_gen_bf16(seed, tensor, count, lo, hi, values);
  return values;
}

static void layer_create(or_model* m, or_layer* L, uint32_t layer_id, int attention) {
  const or_model_config* c = &m->cfg;
  const uint64_t s = c->seed;
  L->attention = attention;
  L->input_norm = bf16_create(s, tensor_id(layer_id, K_INPUT_NORM), c->hidden, -0.1f, 0.1f);
  L->post_norm = bf16_create(s, tensor_id(layer_id, K_POST_NORM), c->hidden, -0.1f, 0.1f);
  matrix_create(&L->gate, s, tensor_id(layer_id, K_GATE), c->intermediate, c->hidden, c->mlp_bits);
  matrix_create(&L->up, s, tensor_id(layer_id, K_UP), c->intermediate, c->hidden, c->mlp_bits);
  matrix_create(&L->down, s, tensor_id(layer_id, K_DOWN), c->hidden, c->intermediate, c->mlp_bits);
  if (attention) {
    matrix_create(&L->q, s, tensor_id(layer_id, K_Q), (size_t)c->q_heads * 512, c->hidden, c->proj_bits);
    matrix_create(&L->k, s, tensor_id(layer_id, K_K), (size_t)c->kv_heads * 256, c->hidden, c->proj_bits);
    matrix_create(&L->v, s, tensor_id(layer_id, K_V), (size_t)c->kv_heads * 256, c->hidden, c->proj_bits);
    matrix_create(&L->out, s, tensor_id(layer_id, K_O), c->hidden, (size_t)c->q_heads * 256, c->proj_bits);
    L->q_norm = bf16_create(s, tensor_id(layer_id, K_QNORM), 256, -0.1f, 0.1f);
    L->k_norm = bf16_create(s, tensor_id(layer_id, K_KNORM), 256, -0.1f, 0.1f);
  } else {
    const size_t channels = (size_t)2 * c->gdn_key_heads * 128 + (size_t)c->gdn_value_heads * 128;
    matrix_create(&L->qkv, s, tensor_id(layer_id, K_QKV), channels, c->hidden, c->proj_bits);
    matrix_create(&L->z, s, tensor_id(layer_id, K_Z), (size_t)c->gdn_value_heads * 128, c->hidden, c->proj_bits);
    matrix_create(&L->a, s, tensor_id(layer_id, K_A), c->gdn_value_heads, c->hidden, c->proj_bits);
    matrix_create(&L->b, s, tensor_id(layer_id, K_B), c->gdn_value_heads, c->hidden, c->proj_bits);
    matrix_create(&L->out, s, tensor_id(layer_id, K_GDN_OUT), c->hidden, (size_t)c->gdn_value_heads * 128, c->proj_bits);
    L->conv = bf16_create(s, tensor_id(layer_id, K_CONV), channels * 4, -0.5f, 0.5f);
    L->a_log = bf16_create(s, tensor_id(layer_id, K_ALOG), c->gdn_value_heads, -1.0f, 1.0f);
    L->dt_bias = bf16_create(s, tensor_id(layer_id, K_DTBIAS), c->gdn_value_heads, -1.0f, 1.0f);
    L->gdn_norm = bf16_create(s, tensor_id(layer_id, K_GDN_NORM), 128, 0.8f, 1.2f);
  }
}

static void layer_free(or_layer* L) {
  free(L->input_norm);
  free(L->post_norm);
  matrix_free(&L->gate);
  matrix_free(&L->up);
  matrix_free(&L->down);
  if (L->attention) {
    matrix_free(&L->q);
    matrix_free(&L->k);
    matrix_free(&L->v);
    free(L->q_norm);
    free(L->k_norm);
  } else {
    matrix_free(&L->qkv);
    matrix_free(&L->z);
    matrix_free(&L->a);
    matrix_free(&L->b);
    free(L->conv);
    free(L->a_log);
    free(L->dt_bias);
    free(L->gdn_norm);
  }
  matrix_free(&L->out);
}

static int is_attention_layer(const or_model_config* c, uint32_t layer) {
  return (layer + 1) % c->attention_interval == 0;
}

static or_model* model_create(const or_model_config* config, int include_mtp, unsigned resident) {
  or_model* m = (or_model*)calloc(1, sizeof(or_model));
  m->cfg = *config;
  m->has_mtp = include_mtp;
  const or_model_config* c = &m->cfg;
  const uint64_t s = c->seed;
  m->resident_layers = resident == 0 || resident > c->layers ? c->layers : resident;
  m->layers = (or_layer*)calloc(c->layers, sizeof(or_layer));
  unsigned gdn_count = 0, attention_count = 0;
  for (uint32_t i = 0; i < c->layers; ++i) {
    const int attention = is_attention_layer(c, i);
    if (i < m->resident_layers) {
      layer_create(m, &m->layers[i], i, attention);
    } else {
      m->layers[i] = m->layers[i % m->resident_layers];
    }
    m->layers[i].state_index = attention ? attention_count++ : gdn_count++;
  }
  matrix_create(&m->embedding, s, tensor_id(LAYER_GLOBAL, G_EMBEDDING), c->vocab, c->hidden, c->emb_bits);
  matrix_create(&m->lm_head, s, tensor_id(LAYER_GLOBAL, G_LM_HEAD), c->vocab, c->hidden, c->head_bits);
  m->final_norm = bf16_create(s, tensor_id(LAYER_GLOBAL, G_FINAL_NORM), c->hidden, -0.1f, 0.1f);
  if (include_mtp) {
    layer_create(m, &m->mtp, LAYER_MTP, 1);
    matrix_create(&m->fc, s, tensor_id(LAYER_MTP, K_FC), c->hidden, (size_t)2 * c->hidden, c->proj_bits);
    m->pre_emb_norm = bf16_create(s, tensor_id(LAYER_MTP, K_PRE_EMB_NORM), c->hidden, -0.1f, 0.1f);
    m->pre_hidden_norm = bf16_create(s, tensor_id(LAYER_MTP, K_PRE_HIDDEN_NORM), c->hidden, -0.1f, 0.1f);
    m->mtp_final_norm = bf16_create(s, tensor_id(LAYER_MTP, K_MTP_FINAL_NORM), c->hidden, -0.1f, 0.1f);
  }
  const size_t channels = (size_t)2 * c->gdn_key_heads * 128 + (size_t)c->gdn_value_heads * 128;
  m->conv_states = (uint16_t*)calloc((size_t)gdn_count * channels * 4, sizeof(uint16_t));
  m->gdn_states = (float*)calloc((size_t)gdn_count * c->gdn_value_heads * 128 * 128, sizeof(float));
  const size_t kv = (size_t)c->kv_heads * 256;
  m->key_caches = (uint16_t*)calloc((size_t)attention_count * c->max_context * kv, sizeof(uint16_t));
  m->value_caches = (uint16_t*)calloc((size_t)attention_count * c->max_context * kv, sizeof(uint16_t));
  m->mtp_keys = (uint16_t*)calloc((size_t)c->max_context * kv, sizeof(uint16_t));
  m->mtp_values = (uint16_t*)calloc((size_t)c->max_context * kv, sizeof(uint16_t));
  m->rope_cos = (float*)malloc((size_t)c->max_context * 32 * sizeof(float));
  m->rope_sin = (float*)malloc((size_t)c->max_context * 32 * sizeof(float));
  or_rope_table(c->max_context, 64, 10000000.0f, m->rope_cos, m->rope_sin);
  const size_t H = c->hidden, I = c->intermediate, B = OR_BLOCK;
  size_t widest = I > channels ? I : channels;
  if ((size_t)c->q_heads * 512 > widest) widest = (size_t)c->q_heads * 512;
  if (2 * H > widest) widest = 2 * H;
  m->widest = widest;
  m->hidden = (uint16_t*)calloc(B * H, 2);
  m->next_hidden = (uint16_t*)calloc(B * H, 2);
  m->normalized = (uint16_t*)calloc(B * H, 2);
  m->post_attention = (uint16_t*)calloc(B * H, 2);
  m->post_normalized = (uint16_t*)calloc(B * H, 2);
  m->last_hidden = (uint16_t*)calloc(H, 2);
  m->mtp_hidden = (uint16_t*)calloc(H, 2);
  m->mtp_input = (uint16_t*)calloc(H, 2);
  m->mtp_concat = (uint16_t*)calloc(2 * H, 2);
  m->conv_out = (uint16_t*)calloc(B * channels, 2);
  m->mixer_out = (uint16_t*)calloc(B * widest, 2);
  m->query = (uint16_t*)calloc(B * c->q_heads * 256, 2);
  m->key = (uint16_t*)calloc(kv, 2);
  m->attn_out = (uint16_t*)calloc(B * c->q_heads * 256, 2);
  m->activated = (uint16_t*)calloc(B * I, 2);
  m->proj_main = (float*)calloc(B * widest, 4);
  m->proj_z = (float*)calloc(B * c->gdn_value_heads * 128, 4);
  m->proj_a = (float*)calloc(B * c->gdn_value_heads, 4);
  m->proj_b = (float*)calloc(B * c->gdn_value_heads, 4);
  m->proj_k = (float*)calloc(B * kv, 4);
  m->proj_v = (float*)calloc(B * kv, 4);
  m->update = (float*)calloc(B * H, 4);
  m->gate = (float*)calloc(B * I, 4);
  m->up = (float*)calloc(B * I, 4);
  m->logits = (float*)calloc(B * (size_t)c->vocab, 4);
  m->last_logits = m->logits;
  m->act_planes = (int8_t*)calloc(B * widest, 1);
  m->act_sums = (int32_t*)calloc(B * (widest / GROUP), 4);
  m->act_scales = (uint16_t*)calloc(B * (widest / GROUP), 2);
  m->act_scale_values = (float*)calloc(B * (widest / GROUP), 4);
  m->act_codes = (int8_t*)calloc(B * widest, 1);
  m->act_packed = (uint8_t*)calloc(B * (widest / 2 + 1), 1);
  return m;
}

or_model* or_model_create(const or_model_config* config, int include_mtp) {
  return model_create(config, include_mtp, 0);
}

/* CPU-baseline model: every layer runs (64 layer applications per token for
 * config 2, each with its own recurrent state and KV cache), but only the
 * first `resident_layers` layers hold weights of their own; layer i reuses
 * those of layer i % resident_layers. The per-token work is the full
 * model's; the host memory is that of `resident_layers` layers. */
or_model* or_model_create_cycled(const or_model_config* config, unsigned resident_layers) {
  return model_create(config, 0, resident_layers);
}

void or_model_destroy(or_model* m) {
  if (!m) return;
  for (uint32_t i = 0; i < m->resident_layers; ++i) layer_free(&m->layers[i]);
  free(m->layers);
  matrix_free(&m->embedding);
  matrix_free(&m->lm_head);
  free(m->final_norm);
  if (m->has_mtp) {
    layer_free(&m->mtp);
    matrix_free(&m->fc);
    free(m->pre_emb_norm);
    free(m->pre_hidden_norm);
    free(m->mtp_final_norm);
  }
  void* buffers[] = {m->conv_states, m->gdn_states, m->key_caches, m->value_caches, m->mtp_keys,
                     m->mtp_values, m->rope_cos, m->rope_sin, m->hidden, m->next_hidden,
                     m->normalized, m->post_attention, m->post_normalized, m->last_hidden,
                     m->mtp_hidden, m->mtp_input, m->mtp_concat, m->conv_out, m->mixer_out,
                     m->query, m->key, m->attn_out, m->activated, m->proj_main, m->proj_z,
                     m->proj_a, m->proj_b, m->proj_k, m->proj_v, m->update, m->gate, m->up,
                     m->logits, m->act_planes, m->act_sums, m->act_scales, m->act_scale_values, m->act_codes,
                     m->act_packed};
  for (size_t i = 0; i < sizeof buffers / sizeof buffers[0]; ++i) free(buffers[i]);
  free(m);
}

static void embed(const or_model* m, uint32_t token, uint16_t* out) {
  const or_matrix* e = &m->embedding;
  const size_t groups = e->columns / GROUP;
  for (size_t c = 0; c < e->columns; ++c) {
    out[c] = or_f32_to_f16((float)matrix_code(e, token, c) *
                           or_f16_to_f32(e->scales[(size_t)token * groups + c / GROUP]));
  }
}

/* q/k/v, Q/K norm + RoPE, KV append, gated attention, o_proj for `count`
 * tokens at positions base .. base + count - 1 (qwen_runtime.cpp:372-404). */
static void attention_block(or_model* m, const or_layer* L, uint16_t* key_cache,
                            uint16_t* value_cache, size_t base, unsigned count) {
  const or_model_config* c = &m->cfg;
  const size_t kv = (size_t)c->kv_heads * 256, qw = (size_t)c->q_heads * 512, qo = (size_t)c->q_heads * 256;
  const size_t H = c->hidden;
  apply_block(m, &L->q, m->normalized, count, m->proj_main);
  apply_block(m, &L->k, m->normalized, count, m->proj_k);
  apply_block(m, &L->v, m->normalized, count, m->proj_v);
  for (unsigned t = 0; t < count; ++t) {
    const size_t position = base + t;
    or_qk_norm_rope(m->proj_main + t * qw, 512, L->q_norm, c->q_heads, position, m->rope_cos, m->rope_sin, 64,
                    m->query + t * qo);
    or_qk_norm_rope(m->proj_k + t * kv, 256, L->k_norm, c->kv_heads, position, m->rope_cos, m->rope_sin, 64,
                    m->key);
    for (size_t i = 0; i < kv; ++i) {
      key_cache[position * kv + i] = m->key[i];
      value_cache[position * kv + i] = or_f32_to_f16(m->proj_v[t * kv + i]);
    }
  }
  for (unsigned t = 0; t < count; ++t) {
    or_gated_attention(m->query + t * qo, m->proj_main + t * qw, key_cache, value_cache, base + t + 1,
                       c->q_heads, c->kv_heads, m->attn_out + t * qo);
  }
  (void)H;
  apply_block(m, &L->out, m->attn_out, count, m->update);
}

static void mlp_block(or_model* m, const or_layer* L, unsigned count) {
  const or_model_config* c = &m->cfg;
  const size_t I = c->intermediate;
  apply_block(m, &L->gate, m->post_normalized, count, m->gate);
  apply_block(m, &L->up, m->post_normalized, count, m->up);
#pragma omp parallel for schedule(static)
  for (int t = 0; t < (int)count; ++t) {
    or_silu_multiply_f16(m->gate + t * I, m->up + t * I, I, m->activated + t * I);
  }
  apply_block(m, &L->down, m->activated, count, m->update);
}

/* One decoder layer over `count` tokens (qwen_runtime.cpp:349-419); m->normalized
 * holds the layer's normalized input, `input` the residual stream. */
static void run_layer(or_model* m, const or_layer* L, const uint16_t* input, uint16_t* output,
                      const uint16_t* next_norm, unsigned count) {
  const or_model_config* c = &m->cfg;
  const float eps = 1.0e-6f;
  const size_t H = c->hidden;
  if (L->attention) {
    const size_t stride = (size_t)c->max_context * c->kv_heads * 256;
    attention_block(m, L, m->key_caches + L->state_index * stride,
                    m->value_caches + L->state_index * stride, m->position, count);
  } else {
    const size_t channels = (size_t)2 * c->gdn_key_heads * 128 + (size_t)c->gdn_value_heads * 128;
    apply_block(m, &L->qkv, m->normalized, count, m->proj_main);
    apply_block(m, &L->z, m->normalized, count, m->proj_z);
    apply_block(m, &L->a, m->normalized, count, m->proj_a);
    apply_block(m, &L->b, m->normalized, count, m->proj_b);
    or_gdn_conv_update(m->proj_main, L->conv, m->conv_states + L->state_index * channels * 4,
                       m->conv_out, NULL, channels, count);
    or_gdn_recurrent(m->conv_out, m->proj_z, m->proj_a, m->proj_b, L->a_log, L->dt_bias,
                     L->gdn_norm,
                     m->gdn_states + (size_t)L->state_index * c->gdn_value_heads * 128 * 128,
                     m->mixer_out, NULL, NULL, NULL, c->gdn_key_heads, c->gdn_value_heads, count);
    apply_block(m, &L->out, m->mixer_out, count, m->update);
  }
#pragma omp parallel for schedule(static)
  for (int t = 0; t < (int)count; ++t) {
    or_residual_add_rms_norm(input + t * H, m->update + t * H, L->post_norm, H, eps, 1,
                             m->post_attention + t * H, m->post_normalized + t * H);
  }
  mlp_block(m, L, count);
#pragma omp parallel for schedule(static)
  for (int t = 0; t < (int)count; ++t) {
    or_residual_add_rms_norm(m->post_attention + t * H, m->update + t * H, next_norm, H, eps, 1,
                             output + t * H, m->normalized + t * H);
  }
}

static double now_seconds(void) {
  struct timespec ts;
  clock_gettime(CLOCK_MONOTONIC, &ts);
  return (double)ts.tv_sec + 1e-9 * (double)ts.tv_nsec;
}

/* The causal forward of `count` <= OR_BLOCK tokens at the current position
 * (qwen_runtime.cpp:1264-1392): heads = 0 skips the LM head (prefill), 1
 * applies it to the last token only, 2 to every token. outputs receives the
 * argmax tokens of the tokens whose head ran (argmax over the full synthetic
 * vocabulary). */
static void forward_block(or_model* m, const uint32_t* tokens, unsigned count, int heads, uint32_t* outputs) {
  const or_model_config* c = &m->cfg;
  const size_t H = c->hidden;
  const double t0 = now_seconds();
#pragma omp parallel for schedule(static)
  for (int t = 0; t < (int)count; ++t) {
    embed(m, tokens[t], m->hidden + t * H);
    or_rms_norm(m->hidden + t * H, m->layers[0].input_norm, H, 1.0e-6f, 1, m->normalized + t * H);
  }
  uint16_t* current = m->hidden;
  uint16_t* next = m->next_hidden;
  for (uint32_t i = 0; i < c->layers; ++i) {
    const uint16_t* next_norm = i + 1 < c->layers ? m->layers[i + 1].input_norm : m->final_norm;
    run_layer(m, &m->layers[i], current, next, next_norm, count);
    uint16_t* swap = current;
    current = next;
    next = swap;
  }
  memcpy(m->last_hidden, current + (size_t)(count - 1) * H, H * sizeof(uint16_t));
  if (current != m->hidden) memcpy(m->hidden, current, (size_t)count * H * sizeof(uint16_t));
  const double t1 = now_seconds();
  if (heads == 2) {
    apply_block(m, &m->lm_head, m->normalized, count, m->logits);
    for (unsigned t = 0; t < count; ++t) outputs[t] = or_argmax(m->logits + (size_t)t * c->vocab, c->vocab);
    m->last_logits = m->logits + (size_t)(count - 1) * c->vocab;
  } else if (heads == 1) {
    apply_block(m, &m->lm_head, m->normalized + (size_t)(count - 1) * H, 1, m->logits);
    outputs[count - 1] = or_argmax(m->logits, c->vocab);
    m->last_logits = m->logits;
  }
  m->head_seconds += now_seconds() - t1;
  m->layer_seconds += t1 - t0;
  m->tokens += count;
  m->position += count;
  m->mtp_chain_active = 0;
}

static int valid_block(const or_model* m, const uint32_t* tokens, size_t count) {
  if (count == 0 || m->position + count > m->cfg.max_context) return 0;
  for (size_t i = 0; i < count; ++i) {
    if (tokens[i] >= m->cfg.vocab) return 0;
  }
  return 1;
}

/* qwen_runtime.cpp:1264-1318. */
int or_model_greedy_step(or_model* m, uint32_t token, uint32_t* next_token) {
  if (!valid_block(m, &token, 1)) return 1;
  forward_block(m, &token, 1, 1, next_token);
  return 0;
}

/* qwen_runtime.cpp:1320-1392: the tokens' argmax outputs, one per token. */
int or_model_block_step(or_model* m, const uint32_t* tokens, unsigned count, uint32_t* outputs) {
  if (count > OR_BLOCK || !valid_block(m, tokens, count)) return 1;
  forward_block(m, tokens, count, 2, outputs);
  return 0;
}

/* A prompt of any length, in layer-major blocks of OR_BLOCK tokens, without
 * the LM head (states, caches and the last hidden state as after stepping
 * each token). */
int or_model_prefill(or_model* m, const uint32_t* tokens, size_t count) {
  if (!valid_block(m, tokens, count)) return 1;
  for (size_t done = 0; done < count; done += OR_BLOCK) {
    const unsigned n = (unsigned)(count - done < OR_BLOCK ? count - done : OR_BLOCK);
    forward_block(m, tokens + done, n, 0, NULL);
  }
  return 0;
}

/* qwen_runtime.cpp:715-867 (launch_mtp_proposal) with a direct token. */
int or_model_mtp_draft(or_model* m, uint32_t token, int use_mtp_hidden, uint32_t* draft) {
  const or_model_config* c = &m->cfg;
  if (!m->has_mtp || token >= c->vocab) return 1;
  const float eps = 1.0e-6f;
  const uint16_t* conditioning = use_mtp_hidden ? m->mtp_hidden : m->last_hidden;
  uint16_t* emb = m->next_hidden;
  embed(m, token, emb);
  or_rms_norm(emb, m->pre_emb_norm, c->hidden, eps, 1, m->mtp_concat);
  or_rms_norm(conditioning, m->pre_hidden_norm, c->hidden, eps, 1, m->mtp_concat + c->hidden);
  apply_block(m, &m->fc, m->mtp_concat, 1, m->update);
  for (size_t i = 0; i < c->hidden; ++i) m->mtp_input[i] = or_f32_to_f16(m->update[i]);
  or_rms_norm(m->mtp_input, m->mtp.input_norm, c->hidden, eps, 1, m->normalized);
  attention_block(m, &m->mtp, m->mtp_keys, m->mtp_values, m->mtp_position, 1);
  or_residual_add_rms_norm(m->mtp_input, m->update, m->mtp.post_norm, c->hidden, eps, 1,
                           m->post_attention, m->post_normalized);
  mlp_block(m, &m->mtp, 1);
  or_residual_add_rms_norm(m->post_attention, m->update, m->mtp_final_norm, c->hidden, eps, 1,
                           m->mtp_hidden, m->normalized);
  const size_t draft_rows = c->draft_vocab < c->vocab ? c->draft_vocab : c->vocab;
  apply_block_rows(m, &m->lm_head, draft_rows, m->normalized, 1, m->logits);
  m->last_logits = m->logits;
  *draft = or_argmax(m->logits, draft_rows);
  m->mtp_position += 1;
  return 0;
}

size_t or_model_position(const or_model* m) { return m->position; }

/* Cumulative seconds spent in the decoder layers and in the LM head + argmax. */
void or_model_timing(const or_model* m, double* layer_seconds, double* head_seconds, size_t* tokens) {
  *layer_seconds = m->layer_seconds;
  *head_seconds = m->head_seconds;
  *tokens = m->tokens;
}

int or_set_threads(int threads) {
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
  return omp_get_max_threads();
#else
  (void)threads;
  return 1;
#endif
}
const uint16_t* or_model_last_hidden(const or_model* m) { return m->last_hidden; }
const float* or_model_logits(const or_model* m) { return m->last_logits; }
