/* Test infrastructure only: plain-C restatement of the reference typed CPU
 * executor (see typed_oracle.h for the reference functions it follows).
 * Compiled by oracle/Makefile with -ffp-contract=off -fno-fast-math so that
 * every float operation below is one IEEE binary32 operation, as
 * docs/reloc-typed-semantics.md §2 requires. */
#include "typed_oracle.h"

#include <math.h>
#include <stdio.h>
#include <string.h>

/* Round-half-even right shift of a non-negative integer by s >= 1 bits. */
static uint32_t rne_shift(uint32_t m, unsigned s) {
  if (s >= 32)
    return 0; /* m < 2^32, so m / 2^s < 1/2 when s >= 33; s == 32 ties only at m == 2^31 */
  uint32_t q = m >> s;
  uint32_t rem = m & ((1u << s) - 1u);
  uint32_t half = 1u << (s - 1);
  if (rem > half || (rem == half && (q & 1u)))
    ++q;
  return q;
}

/* docs/reloc-typed-semantics.md §3.1: binary32 -> binary16, ties to even,
 * subnormals exact, overflow to infinity. NaN: quiet bit plus the top payload
 * bits, the convention of libreloc/quant/Quant.cpp:107-133 (only NaN-ness is
 * normative). */
uint16_t orc_narrow_f16(uint32_t x) {
  const uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
  const uint32_t a = x & 0x7fffffffu;
  if (a > 0x7f800000u)
    return (uint16_t)(sign | 0x7e00u | ((a >> 13) & 0x3ffu));
  if (a == 0x7f800000u)
    return (uint16_t)(sign | 0x7c00u);
  const int biased = (int)(a >> 23);
  const uint32_t frac = a & 0x7fffffu;
  /* significand M and exponent E with value = M * 2^E */
  const uint32_t m = biased ? (frac | 0x800000u) : frac;
  const int e = biased ? biased - 150 : -149;
  if (a < 0x38800000u) {
    /* |x| < 2^-14: the binary16 subnormal grid, quantum 2^-24. */
    const int shift = -24 - e; /* >= 13 */
    return (uint16_t)(sign | rne_shift(m, (unsigned)shift));
  }
  /* Normal binary16 range: keep 11 significant bits. */
  uint32_t r = rne_shift(m, 13);
  int eh = (biased - 127) + 15;
  if (r == 0x800u) { /* rounding carried into the next binade */
    r = 0x400u;
    ++eh;
  }
  if (eh >= 31)
    return (uint16_t)(sign | 0x7c00u);
  return (uint16_t)(sign | ((uint32_t)eh << 10) | (r & 0x3ffu));
}

/* §3.5: binary32 -> bfloat16, ties to even on the discarded 16 bits; the
 * carry runs into the exponent (overflow rounds to infinity). NaN: quiet bit
 * set on the truncated pattern (libreloc/quant/Quant.cpp:164-174). */
uint16_t orc_narrow_bf16(uint32_t x) {
  const uint32_t a = x & 0x7fffffffu;
  if (a > 0x7f800000u)
    return (uint16_t)((x >> 16) | 0x0040u);
  return (uint16_t)(((x >> 16) & 0x8000u) | rne_shift(a, 16));
}

/* §3.2: binary16 -> binary32, exact. */
uint32_t orc_widen_f16(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  const uint32_t exp = (h >> 10) & 0x1fu;
  const uint32_t mant = h & 0x3ffu;
  if (exp == 0) {
    if (mant == 0)
      return sign;
    const float v = ldexpf((float)mant, -24); /* exact: mant < 2^10 */
    uint32_t bits;
    memcpy(&bits, &v, 4);
    return sign | bits;
  }
  if (exp == 31)
    return sign | 0x7f800000u | (mant << 13);
  return sign | ((exp + 112u) << 23) | (mant << 13);
}

/* §3.6: bfloat16 -> binary32, exact. */
uint32_t orc_widen_bf16(uint16_t b) { return (uint32_t)b << 16; }

/* §3.3 step 1: the reciprocal, formed once per parameter element. */
float orc_reciprocal(float scale) { return 1.0f / scale; }

/* §3.3 steps 2-4: one multiply, maxNum(-128) then minNum(127) (NaN -> -128),
 * round half to even. */
int8_t orc_quantize(uint32_t bits, float inv) {
  float x;
  memcpy(&x, &bits, 4);
  float t = x * inv;
  t = fmaxf(t, -128.0f);
  t = fminf(t, 127.0f);
  return (int8_t)nearbyintf(t);
}

/* §3.4: exact integer difference, then one multiply. */
uint32_t orc_dequantize(int8_t q, int32_t zp, float scale) {
  const float d = (float)((int32_t)q - zp);
  const float y = d * scale;
  uint32_t bits;
  memcpy(&bits, &y, 4);
  return bits;
}

static void put(char *err, size_t cap, const char *msg) {
  if (err && cap) {
    strncpy(err, msg, cap - 1);
    err[cap - 1] = 0;
  }
}

static int64_t floordiv64(int64_t a, int64_t b) {
  int64_t q = a / b;
  if ((a % b != 0) && ((a < 0) != (b < 0)))
    --q;
  return q;
}

/* Postfix evaluation of a channel expression over result coordinates. */
static int eval_channel(const orc_stage *s, const orc_program *p,
                        const int64_t *coords, int64_t *out) {
  int64_t stack[ORC_MAX_TOKENS];
  int depth = 0;
  for (int i = 0; i < s->ntokens; ++i) {
    const int op = s->token_op[i];
    const int64_t v = s->token_value[i];
    if (op == 0) {
      if (v < 0 || v >= p->nsymbols)
        return 0;
      stack[depth++] = p->symbols[v];
    } else if (op == 1) {
      stack[depth++] = v;
    } else if (op == 7) {
      if (v < 0 || v >= p->result_rank)
        return 0;
      stack[depth++] = coords[v];
    } else {
      if (depth < 2)
        return 0;
      const int64_t r = stack[--depth];
      const int64_t l = stack[--depth];
      int64_t o;
      switch (op) {
      case 2: o = l + r; break;
      case 3: o = l - r; break;
      case 4: o = l * r; break;
      case 5:
        if (r == 0) return 0;
        o = floordiv64(l, r);
        break;
      case 6:
        if (r == 0) return 0;
        o = l - floordiv64(l, r) * r;
        break;
      default:
        return 0;
      }
      stack[depth++] = o;
    }
  }
  if (depth != 1)
    return 0;
  *out = stack[0];
  return 1;
}

static uint64_t load_bits(const uint8_t *p, int w) {
  uint64_t b = 0;
  memcpy(&b, p, (size_t)w);
  return b;
}

static void store_bits(uint8_t *p, uint64_t b, int w) { memcpy(p, &b, (size_t)w); }

static int run_window(const orc_program *p, const void *srcv, void *dstv,
                      int64_t row_begin, int64_t row_end, char *err,
                      size_t cap) {
  const uint8_t *src = (const uint8_t *)srcv;
  uint8_t *dst = (uint8_t *)dstv;
  const int r = p->rank;
  if (r < 1 || r > ORC_MAX_RANK || p->nstages > ORC_MAX_STAGES) {
    put(err, cap, "unsupported program shape");
    return 1;
  }
  /* Inverse scales, formed once. */
  static float inv_store[ORC_MAX_STAGES][1 << 16];
  const float *inv[ORC_MAX_STAGES] = {0};
  for (int k = 0; k < p->nstages; ++k) {
    const orc_stage *s = &p->stages[k];
    if (s->op == ORC_QUANTIZE) {
      if (s->channel_length > (1 << 16)) {
        put(err, cap, "too many channels for the oracle");
        return 1;
      }
      for (int64_t c = 0; c < s->channel_length; ++c)
        inv_store[k][c] = orc_reciprocal(s->scale[c]);
      inv[k] = inv_store[k];
    }
  }
  int64_t res_strides[ORC_MAX_RANK];
  res_strides[p->result_rank - 1] = 1;
  for (int j = p->result_rank - 1; j > 0; --j)
    res_strides[j - 1] = res_strides[j] * p->result_extents[j];

  /* Window in physical rows of axis 0. */
  int64_t padded0 = p->extents[0] + p->pad_lo[0] + p->pad_hi[0];
  if (row_begin < 0 || row_end > padded0 || row_end < row_begin) {
    put(err, cap, "invalid row window");
    return 1;
  }
  const int64_t origin = row_begin * p->dst_strides[0];
  int64_t window_elems = (row_end - row_begin) * p->dst_strides[0];
  if (row_begin == 0 && row_end == padded0) {
    /* whole result: its size is the product of the padded extents */
    window_elems = 1;
    for (int k = 0; k < r; ++k)
      window_elems *= p->extents[k] + p->pad_lo[k] + p->pad_hi[k];
  }
  if (p->has_fill)
    for (int64_t i = 0; i < window_elems; ++i)
      store_bits(dst + i * p->dst_width, p->fill_bits, p->dst_width);

  int64_t v_begin = row_begin - p->pad_lo[0];
  int64_t v_end = row_end - p->pad_lo[0];
  if (v_begin < 0) v_begin = 0;
  if (v_end > p->extents[0]) v_end = p->extents[0];
  if (v_end <= v_begin)
    return 0;

  int64_t idx[ORC_MAX_RANK] = {0};
  idx[0] = v_begin;
  int64_t coords[ORC_MAX_RANK];
  for (;;) {
    int64_t so = 0, dof = 0;
    for (int k = 0; k < r; ++k) {
      so += idx[k] * p->src_strides[k];
      dof += (idx[k] + p->pad_lo[k]) * p->dst_strides[k];
    }
    uint64_t bits = load_bits(src + so * p->src_width, p->src_width);
    int have_coords = 0;
    for (int k = 0; k < p->nstages; ++k) {
      const orc_stage *s = &p->stages[k];
      int64_t c = 0;
      if (s->per_channel) {
        if (!have_coords) {
          int64_t rest = dof;
          for (int j = 0; j < p->result_rank; ++j) {
            coords[j] = rest / res_strides[j];
            rest -= coords[j] * res_strides[j];
          }
          have_coords = 1;
        }
        if (s->channel_is_dim) {
          c = coords[s->channel_dim];
        } else if (!eval_channel(s, p, coords, &c)) {
          put(err, cap, "channel_evaluation_failed");
          return 1;
        }
        if (c < 0 || c >= s->channel_length) {
          char m[128];
          snprintf(m, sizeof m, "channel_out_of_range: stage %d selected channel %lld of %lld",
                   k, (long long)c, (long long)s->channel_length);
          put(err, cap, m);
          return 1;
        }
      }
      switch (s->op) {
      case ORC_NARROW_F16: bits = orc_narrow_f16((uint32_t)bits); break;
      case ORC_NARROW_BF16: bits = orc_narrow_bf16((uint32_t)bits); break;
      case ORC_WIDEN_F16: bits = orc_widen_f16((uint16_t)bits); break;
      case ORC_WIDEN_BF16: bits = orc_widen_bf16((uint16_t)bits); break;
      case ORC_QUANTIZE:
        bits = (uint8_t)orc_quantize((uint32_t)bits, inv[k][s->per_channel ? c : 0]);
        break;
      case ORC_DEQUANTIZE: {
        int32_t zp = 0;
        if (s->zero_point_count == 1)
          zp = s->zero_point[0];
        else if (s->zero_point_count > 1)
          zp = s->zero_point[c];
        bits = orc_dequantize((int8_t)(uint8_t)bits, zp, s->scale[s->per_channel ? c : 0]);
        break;
      }
      default:
        put(err, cap, "unknown stage op");
        return 1;
      }
    }
    store_bits(dst + (dof - origin) * p->dst_width, bits, p->dst_width);
    /* odometer over the valid box, axis 0 limited to the window */
    int k = r - 1;
    for (; k >= 0; --k) {
      ++idx[k];
      const int64_t lim = k == 0 ? v_end : p->extents[k];
      if (idx[k] < lim)
        break;
      idx[k] = 0;
    }
    if (k < 0)
      break;
  }
  return 0;
}

int orc_execute(const orc_program *p, const void *src, void *dst, char *err,
                size_t cap) {
  const int64_t padded0 = p->extents[0] + p->pad_lo[0] + p->pad_hi[0];
  return run_window(p, src, dst, 0, padded0, err, cap);
}

int orc_execute_rows(const orc_program *p, const void *src, void *dst,
                     int64_t row_begin, int64_t row_end, char *err,
                     size_t cap) {
  return run_window(p, src, dst, row_begin, row_end, err, cap);
}
