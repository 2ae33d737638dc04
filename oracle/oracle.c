/*
 * CPU oracle for the routed-MoE hot path: TEST INFRASTRUCTURE ONLY (see oracle.h).
 *
 * Every function restates the arithmetic of the reference Rust crates at the
 * file:line named in its comment.  Compiled with -ffp-contract=off and without
 * fast-math so that `a * b + c` rounds twice, exactly like Rust's f32 ops.
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------------- */
/* crates/glm-format/src/float.rs:3-73                                        */
/* ------------------------------------------------------------------------- */

static const float kE2m1Positive[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};

/* float.rs:6-13 */
float orc_decode_e2m1(uint8_t code) {
  const float magnitude = kE2m1Positive[code & 0x07];
  return (code & 0x08) == 0 ? magnitude : -magnitude;
}

/* float.rs:15-36: nearest magnitude, ties to the even code. */
int orc_encode_e2m1(float value, uint8_t* code) {
  if (!isfinite(value)) return ORC_ERR_NONFINITE;
  if (value == 0.0f) {
    *code = 0;
    return ORC_OK;
  }
  const uint8_t sign = signbit(value) ? 0x08 : 0;
  const float magnitude = fabsf(value);
  uint8_t best = 0;
  float best_distance = INFINITY;
  for (uint8_t c = 0; c <= 7; ++c) {
    const float distance = fabsf(magnitude - kE2m1Positive[c]);
    if (distance < best_distance ||
        (distance == best_distance && (c & 1) == 0 && (best & 1) == 1)) {
      best = c;
      best_distance = distance;
    }
  }
  *code = sign | best;
  return ORC_OK;
}

/* float.rs:38-50 (2^k computed with ldexpf, which is exact, like powi for these k). */
float orc_decode_e4m3(uint8_t code) {
  const float sign = (code & 0x80) == 0 ? 1.0f : -1.0f;
  const int exponent = (code >> 3) & 0x0f;
  const int mantissa = code & 0x07;
  float magnitude;
  if (exponent == 0) {
    magnitude = (float)mantissa * ldexpf(1.0f, -9);
  } else if (exponent == 15 && mantissa == 7) {
    magnitude = NAN;
  } else {
    magnitude = (1.0f + (float)mantissa / 8.0f) * ldexpf(1.0f, exponent - 7);
  }
  return sign * magnitude;
}

static float g_e4m3_table[127];
static int g_e4m3_ready = 0;

static void e4m3_table_init(void) {
  if (g_e4m3_ready) return;
  for (int c = 0; c <= 0x7e; ++c) g_e4m3_table[c] = orc_decode_e4m3((uint8_t)c);
  g_e4m3_ready = 1;
}

/* float.rs:52-73: nearest over codes 0..=0x7e, ties to the even code. */
int orc_encode_e4m3(float value, uint8_t* code) {
  if (!isfinite(value)) return ORC_ERR_NONFINITE;
  if (value == 0.0f) {
    *code = 0;
    return ORC_OK;
  }
  e4m3_table_init();
  const uint8_t sign = signbit(value) ? 0x80 : 0;
  const float magnitude = fabsf(value);
  uint8_t best = 0;
  float best_distance = INFINITY;
  for (int c = 0; c <= 0x7e; ++c) {
    const float distance = fabsf(magnitude - g_e4m3_table[c]);
    if (distance < best_distance ||
        (distance == best_distance && (c & 1) == 0 && (best & 1) == 1)) {
      best = (uint8_t)c;
      best_distance = distance;
    }
  }
  *code = sign | best;
  return ORC_OK;
}

/* ------------------------------------------------------------------------- */
/* crates/glm-format/src/crc32c.rs:1-13                                       */
/* ------------------------------------------------------------------------- */
uint32_t orc_crc32c(const uint8_t* bytes, uint64_t length) {
  uint32_t crc = ~0u;
  for (uint64_t i = 0; i < length; ++i) {
    crc ^= bytes[i];
    for (int b = 0; b < 8; ++b) {
      const uint32_t mask = 0u - (crc & 1u);
      crc = (crc >> 1) ^ (0x82f63b78u & mask);
    }
  }
  return ~crc;
}

/* ------------------------------------------------------------------------- */
/* crates/glm-format/src/nvfp4.rs                                             */
/* ------------------------------------------------------------------------- */

/* nvfp4.rs:493-521: 128x4 atom swizzle. */
int64_t orc_scale_offset(uint64_t n, uint64_t group, uint64_t padded_n, uint64_t padded_k) {
  if (padded_n % 128 != 0 || padded_k % 64 != 0 || n >= padded_n || group >= padded_k / 16)
    return -1;
  const uint64_t n_block = n / 128, n0 = n % 32, n1 = (n % 128) / 32;
  const uint64_t k_block = group / 4, group_in = group % 4, k_blocks = padded_k / 64;
  return (int64_t)(512 * (n_block * k_blocks + k_block) + 16 * n0 + 4 * n1 + group_in);
}

/* nvfp4.rs:567-573 */
static int quantize_scale(float block_amax, float global_scale, uint8_t* code) {
  if (block_amax == 0.0f) {
    *code = 0;
    return ORC_OK;
  }
  return orc_encode_e4m3((block_amax / 6.0f) / global_scale, code);
}

/* nvfp4.rs:576-608 */
static int encode_block(const float* input, uint64_t logical_n, uint64_t logical_k, uint64_t n,
                        uint64_t group, uint64_t padded_k, uint8_t scale_code, float global_scale,
                        uint8_t* output) {
  const float decoded_scale = orc_decode_e4m3(scale_code) * global_scale;
  for (uint64_t lane = 0; lane < 16; ++lane) {
    const uint64_t k = group * 16 + lane;
    const float value = (n < logical_n && k < logical_k) ? input[n * logical_k + k] : 0.0f;
    uint8_t code = 0;
    if (!(value == 0.0f || scale_code == 0)) {
      const int st = orc_encode_e2m1(value / decoded_scale, &code);
      if (st != ORC_OK) return st;
    }
    const uint64_t linear = n * padded_k + k;
    if ((linear & 1) == 0)
      output[linear / 2] = code;
    else
      output[linear / 2] |= (uint8_t)(code << 4);
  }
  return ORC_OK;
}

/* nvfp4.rs:521-546 (block_scale_1d) */
static int block_scale_1d(const float* input, uint64_t logical_n, uint64_t logical_k, uint64_t n,
                          uint64_t group, float global_scale, uint8_t* code) {
  if (n >= logical_n) {
    *code = 0;
    return ORC_OK;
  }
  const uint64_t start = group * 16;
  const uint64_t end = (start + 16) < logical_k ? (start + 16) : logical_k;
  if (start >= end) {
    *code = 0;
    return ORC_OK;
  }
  float amax = 0.0f;
  for (uint64_t i = n * logical_k + start; i < n * logical_k + end; ++i)
    amax = fmaxf(amax, fabsf(input[i]));
  return quantize_scale(amax, global_scale, code);
}

/* nvfp4.rs:548-565 (block_scale_2d) */
static int block_scale_2d(const float* input, uint64_t logical_n, uint64_t logical_k,
                          uint64_t n_tile, uint64_t group, float global_scale, uint8_t* code) {
  const uint64_t start = group * 16;
  if (start >= logical_k || n_tile >= logical_n) {
    *code = 0;
    return ORC_OK;
  }
  float amax = 0.0f;
  const uint64_t n_end = (n_tile + 16) < logical_n ? (n_tile + 16) : logical_n;
  const uint64_t k_end = (start + 16) < logical_k ? (start + 16) : logical_k;
  for (uint64_t n = n_tile; n < n_end; ++n)
    for (uint64_t k = start; k < k_end; ++k) amax = fmaxf(amax, fabsf(input[n * logical_k + k]));
  return quantize_scale(amax, global_scale, code);
}

static uint64_t align_up(uint64_t v, uint64_t a) { return (v + a - 1) / a * a; }

/* nvfp4.rs:170-273 (PackedNvfp4::pack). values/scales must hold
 * padded_n*padded_k/2 and padded_n*padded_k/16 bytes. */
int orc_nvfp4_pack(const float* input, uint64_t logical_n, uint64_t logical_k, int codec,
                   uint8_t* values, uint8_t* scales, float* global_scale_out,
                   float* global_amax_out) {
  if (logical_n == 0 || logical_k == 0) return ORC_ERR_SHAPE;
  const uint64_t padded_n = align_up(logical_n, 128), padded_k = align_up(logical_k, 64);
  const uint64_t elements = padded_n * padded_k;
  float global_amax = 0.0f;
  for (uint64_t i = 0; i < logical_n * logical_k; ++i) {
    if (!isfinite(input[i])) return ORC_ERR_NONFINITE;
    global_amax = fmaxf(global_amax, fabsf(input[i]));
  }
  const float global_scale = global_amax == 0.0f ? 1.0f : global_amax / (448.0f * 6.0f);
  memset(values, 0, elements / 2);
  memset(scales, 0, elements / 16);
  const uint64_t groups_k = padded_k / 16;
  if (codec == ORC_CODEC_1D) {
    for (uint64_t n = 0; n < padded_n; ++n) {
      for (uint64_t g = 0; g < groups_k; ++g) {
        uint8_t sc;
        int st = block_scale_1d(input, logical_n, logical_k, n, g, global_scale, &sc);
        if (st != ORC_OK) return st;
        scales[orc_scale_offset(n, g, padded_n, padded_k)] = sc;
        st = encode_block(input, logical_n, logical_k, n, g, padded_k, sc, global_scale, values);
        if (st != ORC_OK) return st;
      }
    }
  } else if (codec == ORC_CODEC_2D) {
    for (uint64_t nt = 0; nt < padded_n; nt += 16) {
      for (uint64_t g = 0; g < groups_k; ++g) {
        uint8_t sc;
        int st = block_scale_2d(input, logical_n, logical_k, nt, g, global_scale, &sc);
        if (st != ORC_OK) return st;
        for (uint64_t row = nt; row < nt + 16; ++row) {
          scales[orc_scale_offset(row, g, padded_n, padded_k)] = sc;
          st = encode_block(input, logical_n, logical_k, row, g, padded_k, sc, global_scale,
                            values);
          if (st != ORC_OK) return st;
        }
      }
    }
  } else {
    return ORC_ERR_SHAPE;
  }
  *global_scale_out = global_scale;
  *global_amax_out = global_amax;
  return ORC_OK;
}

/* nvfp4.rs:279-301 (PackedNvfp4::dequantize): (e2m1 * e4m3) * global. */
int orc_nvfp4_dequantize(const uint8_t* values, const uint8_t* scales, float global_scale,
                         uint64_t logical_n, uint64_t logical_k, float* output) {
  const uint64_t padded_n = align_up(logical_n, 128), padded_k = align_up(logical_k, 64);
#pragma omp parallel for schedule(static)
  for (int64_t row = 0; row < (int64_t)logical_n; ++row) {
    for (uint64_t col = 0; col < logical_k; ++col) {
      const uint64_t linear = (uint64_t)row * padded_k + col;
      const uint8_t byte = values[linear / 2];
      const uint8_t code = (linear & 1) == 0 ? (byte & 0x0f) : (byte >> 4);
      const uint8_t scale = scales[orc_scale_offset(row, col / 16, padded_n, padded_k)];
      output[row * logical_k + col] =
          orc_decode_e2m1(code) * orc_decode_e4m3(scale) * global_scale;
    }
  }
  return ORC_OK;
}

static void put_u16(uint8_t* out, int off, uint16_t v) {
  out[off] = (uint8_t)v;
  out[off + 1] = (uint8_t)(v >> 8);
}
static void put_u32(uint8_t* out, int off, uint32_t v) {
  for (int i = 0; i < 4; ++i) out[off + i] = (uint8_t)(v >> (8 * i));
}
static void put_f32(uint8_t* out, int off, float v) {
  uint32_t bits;
  memcpy(&bits, &v, 4);
  put_u32(out, off, bits);
}

/* nvfp4.rs:5-13 */
static const uint8_t kLayoutSourceSha[32] = {
    0x59, 0x8e, 0x05, 0x4b, 0xef, 0x21, 0xed, 0xf9, 0x4b, 0x1f, 0xd6, 0xbb, 0x14, 0x47, 0xcf, 0xa9,
    0xcf, 0xcf, 0x5a, 0x59, 0x07, 0xab, 0x37, 0x01, 0x28, 0x10, 0x24, 0x48, 0xdb, 0xb6, 0xd5, 0x30};
static const uint8_t kQuantPolicySha[32] = {
    0xcd, 0x90, 0x95, 0x79, 0x33, 0x44, 0x05, 0xec, 0xd4, 0xcd, 0x8d, 0x9a, 0x6c, 0x2d, 0xfc, 0xba,
    0x7f, 0x01, 0x24, 0xc4, 0xc4, 0xba, 0x92, 0xbc, 0x40, 0xc9, 0x76, 0xd5, 0x74, 0xbe, 0x05, 0xa3};

/* nvfp4.rs:40-78 (Nvfp4Metadata::encode). */
void orc_nvfp4_metadata_encode(int codec, uint32_t logical_n, uint32_t logical_k,
                               uint32_t padded_n, uint32_t padded_k, float global_scale,
                               float global_amax, uint32_t value_bytes, uint32_t scale_bytes,
                               uint8_t out[128]) {
  memset(out, 0, 128);
  put_u16(out, 0, 0);
  put_u16(out, 2, 1);
  put_u16(out, 4, codec == ORC_CODEC_1D ? 0x0100 : 0x0101);
  out[6] = codec == ORC_CODEC_1D ? 1 : 2;
  out[7] = 1;
  put_u32(out, 8, logical_n);
  put_u32(out, 12, logical_k);
  put_u32(out, 16, padded_n);
  put_u32(out, 20, padded_k);
  put_u16(out, 24, 16);
  put_u16(out, 26, codec == ORC_CODEC_1D ? 1 : 16);
  put_u16(out, 28, 0x1201);
  put_u16(out, 30, 0x1201);
  out[32] = out[33] = out[34] = out[35] = 1;
  put_f32(out, 36, global_scale);
  put_f32(out, 40, global_amax);
  put_u32(out, 44, value_bytes);
  put_u32(out, 48, scale_bytes);
  memcpy(out + 56, kLayoutSourceSha, 32);
  memcpy(out + 88, kQuantPolicySha, 32);
  put_u32(out, 120, orc_crc32c(out, 128));
}

/* ------------------------------------------------------------------------- */
/* crates/glm-reference/src/routed_fc1.rs                                     */
/* ------------------------------------------------------------------------- */

/* routed_fc1.rs:156-163 */
float orc_bf16_round(float value) {
  if (!isfinite(value)) return value;
  uint32_t bits;
  memcpy(&bits, &value, 4);
  const uint32_t bias = 0x7fffu + ((bits >> 16) & 1u);
  bits = (bits + bias) & 0xffff0000u;
  float out;
  memcpy(&out, &bits, 4);
  return out;
}

static float bf16_bits_to_f32(uint16_t b) {
  const uint32_t bits = (uint32_t)b << 16;
  float out;
  memcpy(&out, &bits, 4);
  return out;
}

/* routed_fc1.rs:165-167 (libm expf, as Rust's f32::exp on Linux). */
static float silu(float v) { return v / (1.0f + expf(-v)); }

static int cmp_compacted(const void* a, const void* b) {
  const orc_compacted_route* x = (const orc_compacted_route*)a;
  const orc_compacted_route* y = (const orc_compacted_route*)b;
  if (x->expert != y->expert) return x->expert < y->expert ? -1 : 1;
  if (x->token != y->token) return x->token < y->token ? -1 : 1;
  if (x->slot != y->slot) return x->slot < y->slot ? -1 : 1;
  return 0;
}

/* routed_fc1.rs:20-58: validate, then stable sort by (expert, token, slot). */
int orc_compact_routes(const orc_route* routes, uint64_t count, uint64_t token_count,
                       orc_compacted_route* output) {
  uint8_t* slot_counts = calloc(token_count ? token_count : 1, 1);
  uint8_t* slot_masks = calloc(token_count ? token_count : 1, 1);
  uint64_t* expert_masks = calloc(token_count ? token_count * 4 : 1, 8);
  if (!slot_counts || !slot_masks || !expert_masks) {
    free(slot_counts), free(slot_masks), free(expert_masks);
    return ORC_ERR_ALLOC;
  }
  int status = ORC_OK;
  for (uint64_t i = 0; i < count && status == ORC_OK; ++i) {
    const orc_route r = routes[i];
    if (r.token >= token_count || r.expert >= 256 || r.slot >= 8 || !isfinite(r.weight) ||
        r.weight < 0.0f) {
      status = ORC_ERR_ROUTE;
      break;
    }
    const uint8_t slot_bit = (uint8_t)(1u << r.slot);
    const uint64_t word = r.expert / 64, bit = 1ull << (r.expert % 64);
    if ((slot_masks[r.token] & slot_bit) || (expert_masks[r.token * 4 + word] & bit)) {
      status = ORC_ERR_ROUTE;
      break;
    }
    slot_masks[r.token] |= slot_bit;
    expert_masks[r.token * 4 + word] |= bit;
    if (slot_counts[r.token] == 255) {
      status = ORC_ERR_ROUTE;
      break;
    }
    slot_counts[r.token]++;
    output[i].token = r.token;
    output[i].expert = r.expert;
    output[i].slot = r.slot;
    output[i].pad = 0;
  }
  for (uint64_t t = 0; status == ORC_OK && t < token_count; ++t)
    if (slot_counts[t] > 8) status = ORC_ERR_ROUTE;
  free(slot_counts), free(slot_masks), free(expert_masks);
  if (status != ORC_OK) return status;
  /* Keys are unique (no duplicate (token, slot)), so any sort is the stable sort. */
  qsort(output, count, sizeof(orc_compacted_route), cmp_compacted);
  return ORC_OK;
}

/* One-row PackedNvfp4::pack(row, 1, k, 1D) followed by dequantize(): the only
 * row that carries data is row 0 (rows 1..127 of the padded tensor are zero and
 * never read back), so this performs exactly the row-0 arithmetic of
 * nvfp4.rs:170-301. */
static int nvfp4_row_roundtrip(const float* row, uint64_t k, float* out) {
  float amax = 0.0f;
  for (uint64_t i = 0; i < k; ++i) {
    if (!isfinite(row[i])) return ORC_ERR_NONFINITE;
    amax = fmaxf(amax, fabsf(row[i]));
  }
  const float global_scale = amax == 0.0f ? 1.0f : amax / (448.0f * 6.0f);
  const uint64_t padded_k = align_up(k, 64);
  for (uint64_t g = 0; g < padded_k / 16; ++g) {
    uint8_t sc;
    int st = block_scale_1d(row, 1, k, 0, g, global_scale, &sc);
    if (st != ORC_OK) return st;
    const float decoded_scale = orc_decode_e4m3(sc) * global_scale;
    for (uint64_t lane = 0; lane < 16; ++lane) {
      const uint64_t kk = g * 16 + lane;
      if (kk >= k) break;
      const float value = row[kk];
      uint8_t code = 0;
      if (!(value == 0.0f || sc == 0)) {
        st = orc_encode_e2m1(value / decoded_scale, &code);
        if (st != ORC_OK) return st;
      }
      out[kk] = orc_decode_e2m1(code) * orc_decode_e4m3(sc) * global_scale;
    }
  }
  return ORC_OK;
}

/* routed_fc1.rs:66-105 */
int orc_routed_fc1(const float* activations, uint64_t rows, uint64_t k, const uint8_t* w_values,
                   const uint8_t* w_scales, float w_global, uint64_t n, float* output) {
  if (n % 2 != 0) return ORC_ERR_SHAPE;
  const uint64_t li = n / 2;
  float* w = malloc(sizeof(float) * n * k);
  float* row = malloc(sizeof(float) * k);
  float* act = malloc(sizeof(float) * k);
  if (!w || !row || !act) {
    free(w), free(row), free(act);
    return ORC_ERR_ALLOC;
  }
  orc_nvfp4_dequantize(w_values, w_scales, w_global, n, k, w);
  int status = ORC_OK;
  for (uint64_t r = 0; r < rows && status == ORC_OK; ++r) {
    for (uint64_t i = 0; i < k; ++i) row[i] = orc_bf16_round(activations[r * k + i]);
    status = nvfp4_row_roundtrip(row, k, act);
    if (status != ORC_OK) break;
#pragma omp parallel for schedule(static)
    for (int64_t c = 0; c < (int64_t)li; ++c) {
      float gate = 0.0f, up = 0.0f;
      const float* wg = w + (uint64_t)c * k;
      const float* wu = w + (li + (uint64_t)c) * k;
      for (uint64_t i = 0; i < k; ++i) {
        gate += act[i] * wg[i];
        up += act[i] * wu[i];
      }
      output[r * li + (uint64_t)c] = orc_bf16_round(silu(gate) * up);
    }
  }
  free(w), free(row), free(act);
  return status;
}

/* routed_fc1.rs:112-154: 256-lane strided mul_add then binary tree. */
int orc_routed_fc1_fixed_tree_at(const float* activation, uint64_t k, const uint8_t* w_values,
                                 const uint8_t* w_scales, float w_global, uint64_t n,
                                 uint64_t column, float* output) {
  enum { LANES = 256 };
  if (n % 2 != 0 || column >= n / 2) return ORC_ERR_SHAPE;
  const uint64_t li = n / 2;
  float* w = malloc(sizeof(float) * n * k);
  float* row = malloc(sizeof(float) * k);
  float* in = malloc(sizeof(float) * k);
  if (!w || !row || !in) {
    free(w), free(row), free(in);
    return ORC_ERR_ALLOC;
  }
  orc_nvfp4_dequantize(w_values, w_scales, w_global, n, k, w);
  for (uint64_t i = 0; i < k; ++i) row[i] = orc_bf16_round(activation[i]);
  int status = nvfp4_row_roundtrip(row, k, in);
  if (status == ORC_OK) {
    float gate[LANES], up[LANES];
    for (int lane = 0; lane < LANES; ++lane) {
      gate[lane] = 0.0f;
      up[lane] = 0.0f;
      for (uint64_t i = (uint64_t)lane; i < k; i += LANES) {
        gate[lane] = fmaf(in[i], w[column * k + i], gate[lane]);
        up[lane] = fmaf(in[i], w[(li + column) * k + i], up[lane]);
      }
    }
    for (int stride = 128; stride >= 1; stride /= 2)
      for (int lane = 0; lane < stride; ++lane) {
        gate[lane] += gate[lane + stride];
        up[lane] += up[lane + stride];
      }
    *output = orc_bf16_round(silu(gate[0]) * up[0]);
  }
  free(w), free(row), free(in);
  return status;
}

/* ------------------------------------------------------------------------- */
/* crates/glm-reference/src/routed_fc2.rs                                     */
/* ------------------------------------------------------------------------- */

/* routed_fc2.rs:20-89: per assignment in compacted order, NVFP4 round trip of the
 * K=I_r row, sequential dot, output[token] += route_weight * acc. */
int orc_routed_fc2(const float* activated, const orc_route* routes, uint64_t route_count,
                   uint64_t token_count, uint64_t local_intermediate, uint64_t hidden,
                   const uint16_t* weight_experts, const uint8_t* const* down_values,
                   const uint8_t* const* down_scales, const float* down_globals,
                   uint64_t weight_count, float* output) {
  if (hidden == 0 || local_intermediate == 0) return ORC_ERR_SHAPE;
  orc_compacted_route* comp = malloc(sizeof(orc_compacted_route) * (route_count ? route_count : 1));
  if (!comp) return ORC_ERR_ALLOC;
  int status = orc_compact_routes(routes, route_count, token_count, comp);
  if (status != ORC_OK) {
    free(comp);
    return status;
  }
  memset(output, 0, sizeof(float) * token_count * hidden);
  float* src = malloc(sizeof(float) * local_intermediate);
  float* down = malloc(sizeof(float) * hidden * local_intermediate);
  int current = -1;
  for (uint64_t a = 0; a < route_count && status == ORC_OK; ++a) {
    float weight = NAN;
    for (uint64_t i = 0; i < route_count; ++i)
      if (routes[i].token == comp[a].token && routes[i].expert == comp[a].expert &&
          routes[i].slot == comp[a].slot)
        weight = routes[i].weight;
    int wi = -1;
    for (uint64_t i = 0; i < weight_count; ++i)
      if (weight_experts[i] == comp[a].expert) wi = (int)i;
    if (wi < 0) {
      status = ORC_ERR_SHAPE;
      break;
    }
    if (wi != current) {
      orc_nvfp4_dequantize(down_values[wi], down_scales[wi], down_globals[wi], hidden,
                           local_intermediate, down);
      current = wi;
    }
    status = nvfp4_row_roundtrip(activated + a * local_intermediate, local_intermediate, src);
    if (status != ORC_OK) break;
    float* out = output + (uint64_t)comp[a].token * hidden;
#pragma omp parallel for schedule(static)
    for (int64_t c = 0; c < (int64_t)hidden; ++c) {
      float acc = 0.0f;
      const float* wr = down + (uint64_t)c * local_intermediate;
      for (uint64_t i = 0; i < local_intermediate; ++i) acc += src[i] * wr[i];
      out[c] += weight * acc;
    }
  }
  free(comp), free(src), free(down);
  return status;
}

/* routed_fc2.rs:214-258: residual + sum_rank attention, then + sum_rank (routed + shared),
 * both in rank order.  attention may be NULL (treated as zero). */
int orc_finish_sparse_layer(const float* input_residual, const float* attention,
                            const float* routed, const float* shared, uint32_t ranks,
                            uint64_t elements, float* output) {
  for (uint64_t i = 0; i < elements; ++i) output[i] = input_residual ? input_residual[i] : 0.0f;
  if (attention)
    for (uint32_t r = 0; r < ranks; ++r)
      for (uint64_t i = 0; i < elements; ++i) output[i] += attention[r * elements + i];
  for (uint32_t r = 0; r < ranks; ++r)
    for (uint64_t i = 0; i < elements; ++i)
      output[i] += routed[r * elements + i] + (shared ? shared[r * elements + i] : 0.0f);
  return ORC_OK;
}

/* ------------------------------------------------------------------------- */
/* crates/glm-reference/src/matrix.rs:100-282, crates/glm-cli/src/main.rs     */
/* ------------------------------------------------------------------------- */

static void push_route(orc_route* routes, uint64_t* count, uint64_t token, uint64_t expert,
                       uint64_t slot) {
  routes[*count].token = (uint32_t)token;
  routes[*count].expert = (uint16_t)expert;
  routes[*count].slot = (uint8_t)slot;
  routes[*count].pad = 0;
  routes[*count].weight = 1.0f;
  (*count)++;
}

/* matrix.rs:100-162; cases numbered in ROUTING_CASES order (matrix.rs:8-17). */
int orc_generate_routes(int routing_case, uint64_t token_count, orc_route* routes,
                        uint64_t* count) {
  if (token_count == 0) return ORC_ERR_ROUTE;
  *count = 0;
  switch (routing_case) {
    case 0:
    case 1: {
      const uint64_t expert = routing_case == 0 ? 0 : 255;
      for (uint64_t t = 0; t < token_count; ++t) push_route(routes, count, t, expert, 0);
      break;
    }
    case 2:
      for (uint64_t t = 0; t < token_count; ++t)
        for (uint64_t s = 0; s < 8; ++s) push_route(routes, count, t, (t * 8 + s) % 256, s);
      break;
    case 3:
      for (uint64_t t = 0; t < token_count; ++t) {
        push_route(routes, count, t, 0, 0);
        for (uint64_t s = 1; s < 8; ++s)
          push_route(routes, count, t, 1 + (t * 7 + (s - 1) * 31) % 255, s);
      }
      break;
    case 4: {
      static const uint64_t used[8] = {0, 17, 34, 68, 85, 119, 170, 255};
      for (uint64_t t = 0; t < token_count; ++t)
        for (uint64_t s = 0; s < 8; ++s) push_route(routes, count, t, used[s], s);
      break;
    }
    case 5:
      push_route(routes, count, 0, 7, 0);
      push_route(routes, count, 0, 7, 1);
      break;
    case 6: {
      uint64_t start = *count;
      for (uint64_t t = 0; t < token_count; ++t)
        for (int64_t s = 7; s >= 0; --s)
          push_route(routes, count, t, (t * 8 + (uint64_t)s) % 256, (uint64_t)s);
      for (uint64_t i = start, j = *count - 1; i < j; ++i, --j) {
        orc_route tmp = routes[i];
        routes[i] = routes[j];
        routes[j] = tmp;
      }
      break;
    }
    case 7:
      for (uint64_t t = 0; t < token_count; ++t) {
        const uint64_t slots = (t + 1 == token_count) ? 3 : 8;
        for (uint64_t s = 0; s < slots; ++s)
          push_route(routes, count, t, (t * 11 + s * 29) % 256, s);
      }
      break;
    default:
      return ORC_ERR_ROUTE;
  }
  return ORC_OK;
}

static uint64_t rotl64(uint64_t v, int r) { return (v << r) | (v >> (64 - r)); }

/* matrix.rs:276-282 */
static float deterministic_value(uint64_t index, uint64_t domain) {
  const uint64_t mixed = rotl64((index ^ (domain * 0x9e3779b97f4a7c15ull)) * 0xbf58476d1ce4e5b9ull, 29);
  const int32_t sgn = (int32_t)(mixed >> 40) - (1 << 23);
  return (float)sgn / (float)(1 << 21);
}

/* matrix.rs:164-259; cases numbered in NUMERICAL_CASES order (matrix.rs:19-28). */
int orc_generate_numerical_fixture(int numerical_case, uint64_t rows, uint64_t n, uint64_t k,
                                   float* activations, float* weights) {
  if (rows == 0 || n == 0 || k == 0) return ORC_ERR_SHAPE;
  const uint64_t na = rows * k, nw = n * k;
  memset(activations, 0, sizeof(float) * na);
  memset(weights, 0, sizeof(float) * nw);
  switch (numerical_case) {
    case 0:
      break;
    case 1:
      for (uint64_t i = 0; i < na; ++i) activations[i] = orc_decode_e2m1((uint8_t)(i % 16));
      for (uint64_t i = 0; i < nw; ++i) weights[i] = orc_decode_e2m1((uint8_t)(i % 16));
      break;
    case 2:
      for (uint64_t i = 0; i < na; ++i) activations[i] = (i & 1) == 0 ? 1.0f : -1.0f;
      for (uint64_t g = 0; g * 16 < nw; ++g)
        weights[g * 16] = 6.0f * orc_decode_e4m3((uint8_t)(g % 127));
      weights[0] = 6.0f * 448.0f;
      break;
    case 3: {
      uint32_t bmax_bits = 0x7f7f0000u, bmin_bits = 0x00800000u;
      float bmax, bmin;
      memcpy(&bmax, &bmax_bits, 4);
      memcpy(&bmin, &bmin_bits, 4);
      const float vals[6] = {bmax, -bmax, bmin, -bmin, 1.0f, -1.0f};
      for (uint64_t i = 0; i < na; ++i) activations[i] = vals[i % 6];
      const float tiny = ldexpf(1.0f, -120);
      for (uint64_t i = 0; i < nw; ++i) weights[i] = (i & 1) == 0 ? tiny : -tiny;
      break;
    }
    case 4:
      for (uint64_t i = 0; i < na; ++i) activations[i] = (i & 1) == 0 ? 0.5f : -0.5f;
      for (uint64_t g = 0; g * 16 < nw; ++g) weights[g * 16] = 6.0f * orc_decode_e4m3(1);
      weights[0] = 6.0f * 448.0f;
      break;
    case 5:
      for (uint64_t i = 0; i < na; ++i) activations[i] = deterministic_value(i, 0x51);
      for (uint64_t g = 0; g * 16 < nw; ++g) {
        const uint64_t len = (nw - g * 16) < 16 ? (nw - g * 16) : 16;
        for (uint64_t lane = 0; lane < len; ++lane)
          weights[g * 16 + lane] = deterministic_value(g * 16 + lane, 0xa7) * 0.125f;
        weights[g * 16 + (g % len)] = (g & 1) == 0 ? 256.0f : -256.0f;
      }
      break;
    case 6:
      for (uint64_t i = 0; i < na; ++i) activations[i] = (i & 1) == 0 ? 1.0f : -1.0f;
      for (uint64_t i = 0; i < nw; ++i) weights[i] = (i & 1) == 0 ? -0.75f : 0.75f;
      break;
    case 7:
      for (uint64_t i = 0; i < na; ++i) activations[i] = deterministic_value(i, 0x23);
      for (uint64_t i = 0; i < nw; ++i) weights[i] = deterministic_value(i, 0xd1);
      break;
    default:
      return ORC_ERR_SHAPE;
  }
  return ORC_OK;
}

/* crates/glm-cli/src/main.rs:6064-6078 */
void orc_actual_shape_values(uint64_t n, uint64_t k, float* output) {
  for (uint64_t i = 0; i < n * k; ++i) {
    const uint64_t mixed = rotl64(i * 0x9e3779b97f4a7c15ull, 17);
    const int32_t sgn = (int32_t)((mixed >> 48) & 0xffff) - 32768;
    output[i] = (i % 4093 == 0) ? (float)sgn / 128.0f : (float)sgn / 8192.0f;
  }
}

/* ------------------------------------------------------------------------- */
/* Router: crates/glm-reference/src/manifest.rs:188-194 gives only "FP32 linear,   */
/* sigmoid, group-limited top-8, normalized weights x2.5".  This is the          */
/* project's canonical restatement; the CUDA router computes the same bits.      */
/* ------------------------------------------------------------------------- */

/* exp(x) by Cody-Waite range reduction x = n*ln2 + r (two-constant split of ln2)
 * and the degree-7 Taylor polynomial of e^r in Horner form with fused
 * multiply-adds, then scaling by 2^n.  Defined on [-87, 88]; +inf above, 0 below. */
float orc_router_exp(float x) {
  if (isnan(x)) return x;
  if (x > 88.0f) return INFINITY;
  if (x < -87.0f) return 0.0f;
  const float n = rintf(x * 1.44269502f);
  float r = fmaf(-n, 0.693145751953125f, x);
  r = fmaf(-n, 1.42860677e-06f, r);
  float p = 1.98412701e-04f; /* 1/5040 */
  p = fmaf(p, r, 1.38888892e-03f); /* 1/720 */
  p = fmaf(p, r, 8.33333377e-03f); /* 1/120 */
  p = fmaf(p, r, 4.16666679e-02f); /* 1/24 */
  p = fmaf(p, r, 1.66666672e-01f); /* 1/6 */
  p = fmaf(p, r, 0.5f);
  p = fmaf(p, r, 1.0f);
  p = fmaf(p, r, 1.0f);
  const uint32_t bits = (uint32_t)((int32_t)n + 127) << 23;
  float scale;
  memcpy(&scale, &bits, 4);
  return p * scale;
}

float orc_router_sigmoid(float x) { return 1.0f / (1.0f + orc_router_exp(-x)); }

/* logit[t][e] = ((s_0 + s_1) + ...) + s_7, s_c = fma-chain over the c-th eighth of
 * the hidden dimension in ascending k, starting from 0. */
void orc_router_logits(const uint16_t* x_bf16, uint64_t tokens, uint64_t hidden,
                       const uint16_t* w_bf16, uint64_t experts, float* logits, int threads) {
  const uint64_t chunk = hidden / 8;
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
#else
  (void)threads;
#endif
#pragma omp parallel for schedule(static) collapse(2)
  for (int64_t t = 0; t < (int64_t)tokens; ++t) {
    for (int64_t e = 0; e < (int64_t)experts; ++e) {
      const uint16_t* xr = x_bf16 + (uint64_t)t * hidden;
      const uint16_t* wr = w_bf16 + (uint64_t)e * hidden;
      float total = 0.0f;
      for (uint64_t c = 0; c < 8; ++c) {
        float s = 0.0f;
        for (uint64_t k = c * chunk; k < (c + 1) * chunk; ++k)
          s = fmaf(bf16_bits_to_f32(xr[k]), bf16_bits_to_f32(wr[k]), s);
        total = c == 0 ? s : total + s;
      }
      logits[(uint64_t)t * experts + (uint64_t)e] = total;
    }
  }
}

/* Sigmoid scores s; choice = s + bias; group score = top1 + top2 of choice in the
 * group; keep the best topk_groups groups; take the topk best experts by choice
 * among them (slot order = descending choice, ties -> lower index); weight_i =
 * (s_i / sum_slots s) * route_scale, sum taken in slot order. */
int orc_router_select(const float* logits, uint64_t tokens, uint64_t experts, const float* bias,
                      uint32_t groups, uint32_t topk_groups, uint32_t topk, float route_scale,
                      uint16_t* experts_out, float* weights_out) {
  if (experts == 0 || experts > 256 || groups == 0 || experts % groups != 0 || topk == 0 ||
      topk > 8 || topk_groups == 0 || topk_groups > groups)
    return ORC_ERR_SHAPE;
  const uint64_t gs = experts / groups;
  for (uint64_t t = 0; t < tokens; ++t) {
    float s[256], choice[256], gscore[256];
    int group_on[256], taken[256];
    for (uint64_t e = 0; e < experts; ++e) {
      s[e] = orc_router_sigmoid(logits[t * experts + e]);
      choice[e] = s[e] + bias[e];
      taken[e] = 0;
    }
    for (uint64_t g = 0; g < groups; ++g) {
      float top1 = -INFINITY, top2 = -INFINITY;
      for (uint64_t e = g * gs; e < (g + 1) * gs; ++e) {
        if (choice[e] > top1) {
          top2 = top1;
          top1 = choice[e];
        } else if (choice[e] > top2) {
          top2 = choice[e];
        }
      }
      gscore[g] = gs >= 2 ? top1 + top2 : top1;
      group_on[g] = 0;
    }
    for (uint32_t round = 0; round < topk_groups; ++round) {
      int best = -1;
      for (uint64_t g = 0; g < groups; ++g)
        if (!group_on[g] && (best < 0 || gscore[g] > gscore[best])) best = (int)g;
      group_on[best] = 1;
    }
    float denom = 0.0f;
    float sel_s[8];
    for (uint32_t slot = 0; slot < topk; ++slot) {
      int best = -1;
      for (uint64_t e = 0; e < experts; ++e)
        if (group_on[e / gs] && !taken[e] && (best < 0 || choice[e] > choice[best]))
          best = (int)e;
      if (best < 0) return ORC_ERR_SHAPE;
      taken[best] = 1;
      experts_out[t * topk + slot] = (uint16_t)best;
      sel_s[slot] = s[best];
      denom = slot == 0 ? sel_s[0] : denom + sel_s[slot];
    }
    for (uint32_t slot = 0; slot < topk; ++slot)
      weights_out[t * topk + slot] = (sel_s[slot] / denom) * route_scale;
  }
  return ORC_OK;
}

/* ------------------------------------------------------------------------- */
/* Full rank-local layer: compaction (routed_fc1.rs:20-58), FC1 (routed_fc1.rs:    */
/* 66-105), FC2 weighted scatter in compacted order (routed_fc2.rs:20-89), plus    */
/* the bf16 shared expert (checkpoint.rs:1408-1436 tensors; arithmetic unpinned:    */
/* fp32-accumulated bf16 dots, bf16-rounded SwiGLU, as FC1).                       */
/* ------------------------------------------------------------------------- */
int orc_moe_layer(uint32_t tokens, uint32_t hidden, uint32_t experts, uint32_t local_inter,
                  uint32_t topk, const uint16_t* x_bf16, const uint16_t* route_experts,
                  const float* route_weights, const uint8_t* w13_values,
                  const uint8_t* w13_scales, const float* w13_global, const uint8_t* w2_values,
                  const uint8_t* w2_scales, const float* w2_global,
                  const uint16_t* shared13_bf16, const uint16_t* shared2_bf16,
                  uint32_t shared_inter, const uint32_t* token_subset, uint32_t subset_count,
                  float* routed_out, float* shared_out, int threads) {
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
#else
  (void)threads;
#endif
  const uint64_t H = hidden, I = local_inter, N13 = 2ull * local_inter;
  const uint64_t v13 = N13 * H / 2, s13 = N13 * H / 16, v2 = H * I / 2, s2 = H * I / 16;
  const uint32_t nsel = token_subset ? subset_count : tokens;
  /* out_row[t] = output row of token t, or -1 if not in the subset */
  int64_t* out_row = malloc(sizeof(int64_t) * tokens);
  orc_route* routes = malloc(sizeof(orc_route) * (uint64_t)nsel * topk + 1);
  orc_compacted_route* comp = malloc(sizeof(orc_compacted_route) * (uint64_t)nsel * topk + 1);
  float* w13 = malloc(sizeof(float) * N13 * H);
  float* w2 = malloc(sizeof(float) * H * I);
  float* xrow = malloc(sizeof(float) * H);
  float* act = malloc(sizeof(float) * H);
  const uint64_t IS = shared_inter;
  float* hrow = malloc(sizeof(float) * (I > IS ? I : IS));
  float* src = malloc(sizeof(float) * I);
  if (!out_row || !routes || !comp || !w13 || !w2 || !xrow || !act || !hrow || !src) {
    free(out_row), free(routes), free(comp), free(w13), free(w2), free(xrow), free(act);
    free(hrow), free(src);
    return ORC_ERR_ALLOC;
  }
  for (uint32_t t = 0; t < tokens; ++t) out_row[t] = token_subset ? -1 : (int64_t)t;
  if (token_subset)
    for (uint32_t i = 0; i < subset_count; ++i) out_row[token_subset[i]] = i;
  uint64_t count = 0;
  for (uint32_t i = 0; i < nsel; ++i) {
    const uint32_t t = token_subset ? token_subset[i] : i;
    for (uint32_t s = 0; s < topk; ++s) {
      routes[count].token = t;
      routes[count].expert = route_experts[(uint64_t)t * topk + s];
      routes[count].slot = (uint8_t)s;
      routes[count].pad = 0;
      routes[count].weight = route_weights[(uint64_t)t * topk + s];
      ++count;
    }
  }
  int status = orc_compact_routes(routes, count, tokens, comp);
  if (status == ORC_OK) memset(routed_out, 0, sizeof(float) * nsel * H);
  int64_t current = -1;
  for (uint64_t a = 0; a < count && status == ORC_OK; ++a) {
    const uint32_t e = comp[a].expert, t = comp[a].token;
    if (e >= experts) {
      status = ORC_ERR_ROUTE;
      break;
    }
    if ((int64_t)e != current) {
      orc_nvfp4_dequantize(w13_values + e * v13, w13_scales + e * s13, w13_global[e], N13, H,
                           w13);
      orc_nvfp4_dequantize(w2_values + e * v2, w2_scales + e * s2, w2_global[e], H, I, w2);
      current = e;
    }
    float weight = route_weights[(uint64_t)t * topk + comp[a].slot];
    for (uint64_t k = 0; k < H; ++k) xrow[k] = orc_bf16_round(bf16_bits_to_f32(x_bf16[t * H + k]));
    status = nvfp4_row_roundtrip(xrow, H, act);
    if (status != ORC_OK) break;
#pragma omp parallel for schedule(static)
    for (int64_t c = 0; c < (int64_t)I; ++c) {
      float gate = 0.0f, up = 0.0f;
      const float* wg = w13 + (uint64_t)c * H;
      const float* wu = w13 + (I + (uint64_t)c) * H;
      for (uint64_t k = 0; k < H; ++k) {
        gate += act[k] * wg[k];
        up += act[k] * wu[k];
      }
      hrow[c] = orc_bf16_round(silu(gate) * up);
    }
    status = nvfp4_row_roundtrip(hrow, I, src);
    if (status != ORC_OK) break;
    float* out = routed_out + (uint64_t)out_row[t] * H;
#pragma omp parallel for schedule(static)
    for (int64_t c = 0; c < (int64_t)H; ++c) {
      float acc = 0.0f;
      const float* wr = w2 + (uint64_t)c * I;
      for (uint64_t k = 0; k < I; ++k) acc += src[k] * wr[k];
      out[c] += weight * acc;
    }
  }
  if (status == ORC_OK && shared_out) {
    for (uint32_t i = 0; i < nsel; ++i) {
      const uint32_t t = token_subset ? token_subset[i] : i;
      float* out = shared_out + (uint64_t)i * H;
      if (!shared13_bf16 || !shared2_bf16) {
        memset(out, 0, sizeof(float) * H);
        continue;
      }
#pragma omp parallel for schedule(static)
      for (int64_t c = 0; c < (int64_t)IS; ++c) {
        float gate = 0.0f, up = 0.0f;
        const uint16_t* wg = shared13_bf16 + (uint64_t)c * H;
        const uint16_t* wu = shared13_bf16 + (IS + (uint64_t)c) * H;
        for (uint64_t k = 0; k < H; ++k) {
          const float xv = bf16_bits_to_f32(x_bf16[(uint64_t)t * H + k]);
          gate += xv * bf16_bits_to_f32(wg[k]);
          up += xv * bf16_bits_to_f32(wu[k]);
        }
        hrow[c] = orc_bf16_round(silu(gate) * up);
      }
#pragma omp parallel for schedule(static)
      for (int64_t c = 0; c < (int64_t)H; ++c) {
        float acc = 0.0f;
        const uint16_t* wr = shared2_bf16 + (uint64_t)c * IS;
        for (uint64_t k = 0; k < IS; ++k) acc += hrow[k] * bf16_bits_to_f32(wr[k]);
        out[c] = acc;
      }
    }
  }
  free(out_row), free(routes), free(comp), free(w13), free(w2), free(xrow), free(act);
  free(hrow), free(src);
  return status;
}

/* ------------------------------------------------------------------------- */
/* crates/glm-format/src/exl3.rs:404-601                                       */
/* ------------------------------------------------------------------------- */

/* exl3.rs:534-556 */
float orc_f16_bits_to_f32(uint16_t bits) {
  const uint32_t sign = (uint32_t)(bits & 0x8000) << 16;
  const uint32_t exponent = (bits >> 10) & 0x1f;
  const uint32_t fraction = bits & 0x03ff;
  uint32_t out;
  if (exponent == 0 && fraction == 0) {
    out = sign;
  } else if (exponent == 0) {
    uint32_t significand = fraction, exponent32 = 113;
    while ((significand & 0x0400) == 0) {
      significand <<= 1;
      exponent32 -= 1;
    }
    out = sign | (exponent32 << 23) | ((significand & 0x03ff) << 13);
  } else if (exponent == 31) {
    out = sign | 0x7f800000u | (fraction << 13);
  } else {
    out = sign | ((exponent + 112) << 23) | (fraction << 13);
  }
  float f;
  memcpy(&f, &out, 4);
  return f;
}

/* exl3.rs:558-601 */
uint16_t orc_f32_to_f16_bits(float value) {
  uint32_t bits;
  memcpy(&bits, &value, 4);
  const uint16_t sign = (uint16_t)((bits >> 16) & 0x8000);
  const int32_t exponent = (int32_t)((bits >> 23) & 0xff);
  const uint32_t fraction = bits & 0x007fffff;
  if (exponent == 255)
    return sign | (fraction == 0 ? 0x7c00 : (uint16_t)(0x7e00 | ((fraction >> 13) & 0x01ff)));
  const int32_t he = exponent - 127 + 15;
  if (he >= 31) return sign | 0x7c00;
  if (he <= 0) {
    if (he < -10) return sign;
    const uint32_t significand = fraction | 0x00800000u;
    const uint32_t shift = (uint32_t)(14 - he);
    uint32_t rounded = significand >> shift;
    const uint32_t remainder = significand & ((1u << shift) - 1);
    const uint32_t halfway = 1u << (shift - 1);
    if (remainder > halfway || (remainder == halfway && (rounded & 1) != 0)) rounded += 1;
    return sign | (uint16_t)rounded;
  }
  uint32_t rf = fraction >> 13;
  const uint32_t remainder = fraction & 0x1fff;
  if (remainder > 0x1000 || (remainder == 0x1000 && (rf & 1) != 0)) {
    rf += 1;
    if (rf == 0x400) {
      const int32_t ne = he + 1;
      if (ne >= 31) return sign | 0x7c00;
      return sign | (uint16_t)(ne << 10);
    }
  }
  return sign | (uint16_t)(he << 10) | (uint16_t)rf;
}

/* exl3.rs:667-684 (test fixture generator: xorshift 13/7/17, low 16 bits). */
void orc_exl3_xorshift_trellis(uint64_t seed, uint64_t words, uint16_t* trellis) {
  uint64_t state = seed;
  for (uint64_t i = 0; i < words; ++i) {
    state ^= state << 13;
    state ^= state >> 7;
    state ^= state << 17;
    trellis[i] = (uint16_t)state;
  }
}

/* exl3.rs:471-477 */
static uint16_t decode_3inst_f16_direct(uint16_t window) {
  const uint32_t value = (uint32_t)window * 0xCBAC1FEDu;
  const uint32_t packed = (value & 0x8FFF8FFFu) ^ 0x3B603B60u;
  return orc_f32_to_f16_bits(orc_f16_bits_to_f32((uint16_t)packed) +
                             orc_f16_bits_to_f32((uint16_t)(packed >> 16)));
}

/* The decode is a pure function of the 16-bit window: tabulated once. */
static uint16_t g_3inst_table[65536];
static int g_3inst_ready = 0;

static uint16_t decode_3inst_f16(uint16_t window) {
  if (!__atomic_load_n(&g_3inst_ready, __ATOMIC_ACQUIRE)) {
#pragma omp critical(orc_3inst_table)
    if (!g_3inst_ready) {
      for (uint32_t w = 0; w < 65536; ++w) g_3inst_table[w] = decode_3inst_f16_direct((uint16_t)w);
      __atomic_store_n(&g_3inst_ready, 1, __ATOMIC_RELEASE);
    }
  }
  return g_3inst_table[window];
}

/* exl3.rs:479-513 */
uint16_t orc_exl3_decode_native_at(const uint16_t* trellis, uint64_t logical_n, uint32_t bits,
                                   uint64_t row, uint64_t column) {
  const uint64_t tile_halves = 16ull * bits, tile_words = 8ull * bits;
  const uint64_t tile_index = (row / 16) * (logical_n / 16) + column / 16;
  const uint64_t tile_base = tile_index * tile_halves;
  const uint64_t lr = row & 15, lc = column & 15;
  const uint64_t row_quadrant = (lr & 7) >> 1;
  const uint64_t row_selector = (lr >= 8 ? 2 : 0) + (lr & 1);
  const uint64_t column_group = (lc >> 1) & 3, parity = lc & 1;
  const uint64_t lane = column_group * 8 + parity * 4 + row_quadrant;
  const uint64_t weight = (lc >= 8 ? 4 : 0) + row_selector;
  const uint64_t end_bit = (lane * 8 + weight + 257) * bits;
  const uint64_t start_bit = end_bit - 16;
  const uint64_t first_word = start_bit / 32, last_word = (end_bit - 1) / 32;
  const uint64_t shift = (last_word + 1) * 32 - end_bit;
#define READ_WORD(index)                                                   \
  ((uint32_t)trellis[tile_base + ((index) % tile_words) * 2] |             \
   ((uint32_t)trellis[tile_base + ((index) % tile_words) * 2 + 1] << 16))
  const uint64_t merged = ((uint64_t)READ_WORD(first_word) << 32) | (uint64_t)READ_WORD(last_word);
#undef READ_WORD
  return decode_3inst_f16((uint16_t)((merged >> shift) & 0xffff));
}

void orc_exl3_reconstruct_native(const uint16_t* trellis, uint64_t k, uint64_t n, uint32_t bits,
                                 uint16_t* output) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < (int64_t)k; ++r)
    for (uint64_t c = 0; c < n; ++c)
      output[(uint64_t)r * n + c] = orc_exl3_decode_native_at(trellis, n, bits, (uint64_t)r, c);
}

/* exl3.rs:515-531 */
static void hadamard_128(const float* input, float* output) {
  const float normalization = 1.0f / sqrtf(128.0f);
  for (int row = 0; row < 128; ++row) {
    float sum = 0.0f;
    for (int col = 0; col < 128; ++col) {
      const float sign = (__builtin_popcount((unsigned)(row & col)) & 1) == 0 ? 1.0f : -1.0f;
      sum += sign * input[col];
    }
    output[row] = sum * normalization;
  }
}

static float f16_round(float v) { return orc_f16_bits_to_f32(orc_f32_to_f16_bits(v)); }

/* Columns per SIMD block of the fast oracle paths below. */
enum { kPrepCols = 32 };

/* sums of kPrepCols columns [c0, c0 + kPrepCols) over ascending k (defined below). */
static void dot_block(const float* act, uint64_t k_len, const float* wt, uint64_t ld,
                      uint64_t c0, float* out);

/* The decoded weights of one trellis (exl3.rs:490-513), converted once to fp32,
 * [k][n] row-major: the prepared form of an EXL3 projection. */
int orc_exl3_prepare(const uint16_t* trellis, uint64_t k, uint64_t n, uint32_t bits,
                     float* nativef) {
  if (k % 128 != 0 || n % 128 != 0) return ORC_ERR_SHAPE;
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < (int64_t)k; ++r)
    for (uint64_t c = 0; c < n; ++c)
      nativef[(uint64_t)r * n + c] =
          orc_f16_bits_to_f32(orc_exl3_decode_native_at(trellis, n, bits, (uint64_t)r, c));
  return ORC_OK;
}

/* exl3.rs:404-453 (Exl3Trellis::matmul_reference_f16) on prepared weights.
 * Arithmetic per output column is the reference's: an fp32 sum over ascending k
 * of source[k] * w[k][c] (each product and add rounded once), rounded to fp16.
 * For speed all rows' rotated sources are built first and 32 adjacent columns
 * advance together in SIMD lanes. */
int orc_exl3_project(const float* nativef, uint64_t k, uint64_t n, const uint16_t* suh,
                     const uint16_t* svh, const uint16_t* activations, uint64_t rows,
                     uint16_t* output, int threads) {
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
#else
  (void)threads;
#endif
  if (k % 128 != 0 || n % 128 != 0) return ORC_ERR_SHAPE;
  if (rows == 0) return ORC_OK;
  float* source = malloc(sizeof(float) * k * rows);
  float* projected = malloc(sizeof(float) * n * rows);
  if (!source || !projected) {
    free(source), free(projected);
    return ORC_ERR_ALLOC;
  }
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < (int64_t)rows; ++r) {
    float tmp[128];
    float* src = source + (uint64_t)r * k;
    for (uint64_t i = 0; i < k; ++i)
      src[i] = f16_round(orc_f16_bits_to_f32(activations[(uint64_t)r * k + i]) *
                         orc_f16_bits_to_f32(suh[i]));
    for (uint64_t b = 0; b < k; b += 128) {
      hadamard_128(src + b, tmp);
      for (int i = 0; i < 128; ++i) src[b + i] = f16_round(tmp[i]);
    }
  }
  const int64_t tiles = (int64_t)(n / kPrepCols);
#pragma omp parallel for schedule(static) collapse(2)
  for (int64_t r = 0; r < (int64_t)rows; ++r)
    for (int64_t j = 0; j < tiles; ++j) {
      float acc[kPrepCols];
      const uint64_t c0 = (uint64_t)j * kPrepCols;
      dot_block(source + (uint64_t)r * k, k, nativef, n, c0, acc);
      for (int c = 0; c < kPrepCols; ++c) projected[(uint64_t)r * n + c0 + c] = f16_round(acc[c]);
    }
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < (int64_t)rows; ++r) {
    float tmp[128];
    float* pr = projected + (uint64_t)r * n;
    for (uint64_t b = 0; b < n; b += 128) {
      hadamard_128(pr + b, tmp);
      for (int i = 0; i < 128; ++i) pr[b + i] = f16_round(tmp[i] * orc_f16_bits_to_f32(svh[b + i]));
    }
    for (uint64_t c = 0; c < n; ++c) output[(uint64_t)r * n + c] = orc_f32_to_f16_bits(pr[c]);
  }
  free(source), free(projected);
  return ORC_OK;
}

/* exl3.rs:404-453 (Exl3Trellis::matmul_reference_f16): decode, then project. */
int orc_exl3_matmul_reference(const uint16_t* trellis, uint64_t k, uint64_t n, uint32_t bits,
                              const uint16_t* suh, const uint16_t* svh,
                              const uint16_t* activations, uint64_t rows, uint16_t* output,
                              int threads) {
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
#endif
  if (k % 128 != 0 || n % 128 != 0) return ORC_ERR_SHAPE;
  float* nativef = malloc(sizeof(float) * k * n);
  if (!nativef) return ORC_ERR_ALLOC;
  int status = orc_exl3_prepare(trellis, k, n, bits, nativef);
  if (status == ORC_OK)
    status = orc_exl3_project(nativef, k, n, suh, svh, activations, rows, output, threads);
  free(nativef);
  return status;
}

/* ------------------------------------------------------------------------- */
/* Prepared-expert form of orc_moe_layer: the same arithmetic bit for bit,     */
/* arranged for speed as the CPU-baseline plan asks (each expert dequantised    */
/* once, OpenMP over assignments, SIMD across output columns).  Each expert's   */
/* weights are dequantised (nvfp4.rs:279-301) into k-major fp32 planes, so a    */
/* block of output columns keeps one running sum per column in SIMD lanes while */
/* k ascends: every column is still the sequential sum of routed_fc1.rs:84-103  */
/* and routed_fc2.rs:60-86, each product and each add rounded once.            */
/* ------------------------------------------------------------------------- */


static int omp_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* Transpose src [n][k] into dst [k][ld] (blocked). */
static void transpose_into(const float* src, uint64_t n, uint64_t k, float* dst, uint64_t ld) {
#pragma omp parallel for schedule(static) collapse(2)
  for (int64_t nb = 0; nb < (int64_t)((n + 31) / 32); ++nb)
    for (int64_t kb = 0; kb < (int64_t)((k + 31) / 32); ++kb)
      for (uint64_t r = (uint64_t)nb * 32; r < n && r < (uint64_t)nb * 32 + 32; ++r)
        for (uint64_t c = (uint64_t)kb * 32; c < k && c < (uint64_t)kb * 32 + 32; ++c)
          dst[c * ld + r] = src[r * k + c];
}

/* PackedNvfp4::dequantize (nvfp4.rs:279-301, (e2m1 * e4m3) * global, that
 * product order) of an [n][k] tensor written k-major into dst [k][n]: the 16
 * values of a scale block come from a 16-entry table built with the same two
 * products, so every weight is the same float as orc_nvfp4_dequantize's. */
static void dequantize_transposed(const uint8_t* values, const uint8_t* scales,
                                  float global_scale, uint64_t n, uint64_t k, float* dst) {
  const uint64_t padded_n = align_up(n, 128), padded_k = align_up(k, 64);
#pragma omp parallel for schedule(static) collapse(2)
  for (int64_t nb = 0; nb < (int64_t)(n / 64); ++nb)
    for (int64_t kb = 0; kb < (int64_t)(k / 64); ++kb) {
      float tile[64][65];
      for (uint64_t r = 0; r < 64; ++r) {
        const uint64_t row = (uint64_t)nb * 64 + r;
        for (uint64_t g = 0; g < 4; ++g) {
          const uint64_t col0 = (uint64_t)kb * 64 + g * 16;
          const float dec = orc_decode_e4m3(
              scales[orc_scale_offset(row, col0 / 16, padded_n, padded_k)]);
          float lut[16];
          for (int c = 0; c < 16; ++c) lut[c] = orc_decode_e2m1((uint8_t)c) * dec * global_scale;
          const uint8_t* v = values + (row * padded_k + col0) / 2;
          for (int j = 0; j < 8; ++j) {
            tile[r][g * 16 + 2 * j] = lut[v[j] & 0x0f];
            tile[r][g * 16 + 2 * j + 1] = lut[v[j] >> 4];
          }
        }
      }
      for (uint64_t c = 0; c < 64; ++c)
        for (uint64_t r = 0; r < 64; ++r)
          dst[((uint64_t)kb * 64 + c) * n + (uint64_t)nb * 64 + r] = tile[r][c];
    }
}

int orc_expert_prepare(const uint8_t* w13_values, const uint8_t* w13_scales, float w13_global,
                       const uint8_t* w2_values, const uint8_t* w2_scales, float w2_global,
                       uint32_t hidden, uint32_t local_inter, float* w13t, float* w2t) {
  const uint64_t H = hidden, I = local_inter, N13 = 2ull * I;
  if (I % 64 != 0 || H % 64 != 0) return ORC_ERR_SHAPE;
  dequantize_transposed(w13_values, w13_scales, w13_global, N13, H, w13t);
  dequantize_transposed(w2_values, w2_scales, w2_global, H, I, w2t);
  return ORC_OK;
}

int orc_shared_prepare(const uint16_t* shared13_bf16, const uint16_t* shared2_bf16,
                       uint32_t hidden, uint32_t shared_inter, float* s13t, float* s2t) {
  const uint64_t H = hidden, IS = shared_inter, N13 = 2ull * IS;
  if (IS % kPrepCols != 0 || H % kPrepCols != 0) return ORC_ERR_SHAPE;
  float* tmp = malloc(sizeof(float) * N13 * H);
  if (!tmp) return ORC_ERR_ALLOC;
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < (int64_t)(N13 * H); ++i) tmp[i] = bf16_bits_to_f32(shared13_bf16[i]);
  transpose_into(tmp, N13, H, s13t, N13);
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < (int64_t)(H * IS); ++i) tmp[i] = bf16_bits_to_f32(shared2_bf16[i]);
  transpose_into(tmp, H, IS, s2t, H);
  free(tmp);
  return ORC_OK;
}

/* gate/up sums of kPrepCols columns [c0, c0 + kPrepCols) over ascending k. */
__attribute__((target_clones("avx512f", "avx2", "default")))
static void dual_dot_block(const float* act, uint64_t k_len, const float* wt, uint64_t ld,
                           uint64_t c0, uint64_t up_off, float* gate, float* up) {
  float g[kPrepCols], u[kPrepCols];
  for (int c = 0; c < kPrepCols; ++c) g[c] = 0.0f, u[c] = 0.0f;
  for (uint64_t k = 0; k < k_len; ++k) {
    const float a = act[k];
    const float* wk = wt + k * ld + c0;
    for (int c = 0; c < kPrepCols; ++c) g[c] = g[c] + a * wk[c];
    for (int c = 0; c < kPrepCols; ++c) u[c] = u[c] + a * wk[up_off + c];
  }
  for (int c = 0; c < kPrepCols; ++c) gate[c] = g[c], up[c] = u[c];
}

/* sums of kPrepCols columns [c0, c0 + kPrepCols) over ascending k. */
__attribute__((target_clones("avx512f", "avx2", "default")))
static void dot_block(const float* act, uint64_t k_len, const float* wt, uint64_t ld,
                      uint64_t c0, float* out) {
  float s[kPrepCols];
  for (int c = 0; c < kPrepCols; ++c) s[c] = 0.0f;
  for (uint64_t k = 0; k < k_len; ++k) {
    const float a = act[k];
    const float* wk = wt + k * ld + c0;
    for (int c = 0; c < kPrepCols; ++c) s[c] = s[c] + a * wk[c];
  }
  for (int c = 0; c < kPrepCols; ++c) out[c] = s[c];
}

/* FC1 + SwiGLU of one expert's assignments (routed_fc1.rs:84-103): row i is
 * token tokens[i]; h [rows][I] receives bf16_round(silu(gate) * up). */
int orc_moe_expert_h(uint32_t hidden, uint32_t local_inter, const uint16_t* x_bf16,
                     const uint32_t* tokens, uint32_t rows, const float* w13t, float* h,
                     int threads) {
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
#else
  (void)threads;
#endif
  const uint64_t H = hidden, I = local_inter, N13 = 2ull * I;
  if (rows == 0) return ORC_OK;
  if (I % kPrepCols != 0 || H % kPrepCols != 0) return ORC_ERR_SHAPE;
  float* act = malloc(sizeof(float) * rows * H);
  if (!act) return ORC_ERR_ALLOC;
  int status = ORC_OK;
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < (int64_t)rows; ++i) {
    float* ar = act + (uint64_t)i * H;
    float* row = malloc(sizeof(float) * H);
    int st = row ? ORC_OK : ORC_ERR_ALLOC;
    if (st == ORC_OK) {
      for (uint64_t k = 0; k < H; ++k)
        row[k] = orc_bf16_round(bf16_bits_to_f32(x_bf16[(uint64_t)tokens[i] * H + k]));
      st = nvfp4_row_roundtrip(row, H, ar);
    }
    free(row);
    if (st != ORC_OK) {
#pragma omp critical
      status = st;
    }
  }
  if (status == ORC_OK) {
    const int64_t tiles = (int64_t)(I / kPrepCols);
#pragma omp parallel for schedule(dynamic, 1) collapse(2)
    for (int64_t i = 0; i < (int64_t)rows; ++i)
      for (int64_t j = 0; j < tiles; ++j) {
        float gate[kPrepCols], up[kPrepCols];
        const uint64_t c0 = (uint64_t)j * kPrepCols;
        dual_dot_block(act + (uint64_t)i * H, H, w13t, N13, c0, I, gate, up);
        for (int c = 0; c < kPrepCols; ++c)
          h[(uint64_t)i * I + c0 + c] = orc_bf16_round(silu(gate[c]) * up[c]);
      }
  }
  free(act);
  return status;
}

/* One expert's assignments (routed_fc1.rs:84-103 then routed_fc2.rs:60-86):
 * row i is token tokens[i] with routing weight weights[i]; its weighted FC2
 * output is added to out + out_rows[i] * hidden.  Tokens are distinct within an
 * expert, so rows write disjoint outputs; calling this per expert in ascending
 * order keeps the reference's compacted accumulation order. */
int orc_moe_expert_rows(uint32_t hidden, uint32_t local_inter, const uint16_t* x_bf16,
                        const uint32_t* tokens, const float* weights, const uint32_t* out_rows,
                        uint32_t rows, const float* w13t, const float* w2t, float* out,
                        int threads) {
  const uint64_t H = hidden, I = local_inter;
  if (rows == 0) return ORC_OK;
  float* h = malloc(sizeof(float) * rows * I);
  float* src = malloc(sizeof(float) * rows * I);
  if (!h || !src) {
    free(h), free(src);
    return ORC_ERR_ALLOC;
  }
  int status = orc_moe_expert_h(hidden, local_inter, x_bf16, tokens, rows, w13t, h, threads);
  if (status != ORC_OK) goto done;
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < (int64_t)rows; ++i) {
    const int st = nvfp4_row_roundtrip(h + (uint64_t)i * I, I, src + (uint64_t)i * I);
    if (st != ORC_OK) {
#pragma omp critical
      status = st;
    }
  }
  if (status != ORC_OK) goto done;
  {
    const int64_t tiles = (int64_t)(H / kPrepCols);
#pragma omp parallel for schedule(dynamic, 4) collapse(2)
    for (int64_t i = 0; i < (int64_t)rows; ++i)
      for (int64_t j = 0; j < tiles; ++j) {
        float acc[kPrepCols];
        const uint64_t c0 = (uint64_t)j * kPrepCols;
        dot_block(src + (uint64_t)i * I, I, w2t, H, c0, acc);
        float* o = out + (uint64_t)out_rows[i] * H + c0;
        const float weight = weights[i];
        for (int c = 0; c < kPrepCols; ++c) o[c] += weight * acc[c];
      }
  }
done:
  free(h), free(src);
  return status;
}

/* The bf16 shared expert of orc_moe_layer on prepared planes: shared_out row i
 * (token tokens[i]) = down(bf16_round(silu(gate) * up)), sequential-k sums. */
int orc_shared_rows(uint32_t hidden, uint32_t shared_inter, const uint16_t* x_bf16,
                    const uint32_t* tokens, uint32_t rows, const float* s13t, const float* s2t,
                    float* shared_out, int threads) {
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
#else
  (void)threads;
#endif
  const uint64_t H = hidden, IS = shared_inter, N13 = 2ull * IS;
  if (rows == 0) return ORC_OK;
  if (IS % kPrepCols != 0 || H % kPrepCols != 0) return ORC_ERR_SHAPE;
  float* xs = malloc(sizeof(float) * rows * H);
  float* h = malloc(sizeof(float) * rows * IS);
  if (!xs || !h) {
    free(xs), free(h);
    return ORC_ERR_ALLOC;
  }
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < (int64_t)rows; ++i)
    for (uint64_t k = 0; k < H; ++k)
      xs[(uint64_t)i * H + k] = bf16_bits_to_f32(x_bf16[(uint64_t)tokens[i] * H + k]);
  {
    const int64_t tiles = (int64_t)(IS / kPrepCols);
#pragma omp parallel for schedule(dynamic, 1) collapse(2)
    for (int64_t i = 0; i < (int64_t)rows; ++i)
      for (int64_t j = 0; j < tiles; ++j) {
        float gate[kPrepCols], up[kPrepCols];
        const uint64_t c0 = (uint64_t)j * kPrepCols;
        dual_dot_block(xs + (uint64_t)i * H, H, s13t, N13, c0, IS, gate, up);
        for (int c = 0; c < kPrepCols; ++c)
          h[(uint64_t)i * IS + c0 + c] = orc_bf16_round(silu(gate[c]) * up[c]);
      }
  }
  {
    const int64_t tiles = (int64_t)(H / kPrepCols);
#pragma omp parallel for schedule(dynamic, 4) collapse(2)
    for (int64_t i = 0; i < (int64_t)rows; ++i)
      for (int64_t j = 0; j < tiles; ++j) {
        const uint64_t c0 = (uint64_t)j * kPrepCols;
        dot_block(h + (uint64_t)i * IS, IS, s2t, H, c0, shared_out + (uint64_t)i * H + c0);
      }
  }
  free(xs), free(h);
  return ORC_OK;
}

int orc_threads(void) { return omp_threads(); }
