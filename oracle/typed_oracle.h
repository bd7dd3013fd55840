/* Test infrastructure only: a plain-C restatement of the reference's typed
 * CPU executor, used by the parity tests as an independent checker of the
 * CUDA path. Never linked by the product.
 *
 * The restated algorithm is libreloc's typed::executeHost
 * (libreloc/src/TypedExecute.cpp:727-922): fill every destination element
 * with the fused pad fill, then walk the valid cells of the coalesced layout
 * (walk, :223-260), applying the value stages in order to each element
 * (applyStage, :472-499) with per-channel parameters selected by the logical
 * result coordinate decoded from the destination offset (element, :182-221).
 * The scalar arithmetic follows docs/reloc-typed-semantics.md §3.
 */
#ifndef SYM_B200_TYPED_ORACLE_H
#define SYM_B200_TYPED_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#define ORC_MAX_RANK 8
#define ORC_MAX_STAGES 8
#define ORC_MAX_TOKENS 64
#define ORC_MAX_SYMBOLS 32

enum orc_stage_op {
  ORC_NARROW_F16 = 0,  /* cast f32 -> f16, ieee_rne */
  ORC_NARROW_BF16 = 1, /* cast f32 -> bf16, ieee_rne */
  ORC_WIDEN_F16 = 2,   /* cast f16 -> f32, exact */
  ORC_WIDEN_BF16 = 3,  /* cast bf16 -> f32, exact */
  ORC_QUANTIZE = 4,    /* f32 -> s8, symmetric_rne */
  ORC_DEQUANTIZE = 5   /* s8 -> f32, affine */
};

typedef struct {
  int32_t op;
  int32_t per_channel;    /* 0: one parameter for every element */
  int32_t channel_is_dim; /* 1: channel = result coordinate channel_dim */
  int32_t channel_dim;
  int64_t channel_length; /* parameter entries */
  const float *scale;     /* declared scales (the oracle forms 1/scale) */
  const int32_t *zero_point;
  int64_t zero_point_count; /* 0 = absent (0), 1 = broadcast, else per channel */
  /* Channel expression in wire postfix form (PUSH_SYM 0, PUSH_CONST 1,
   * ADD 2, SUB 3, MUL 4, FLOORDIV 5, MOD 6, PUSH_DIM 7), used when
   * channel_is_dim is 0. */
  int32_t ntokens;
  int32_t token_op[ORC_MAX_TOKENS];
  int64_t token_value[ORC_MAX_TOKENS];
} orc_stage;

typedef struct {
  int32_t rank; /* coalesced layout rank */
  int64_t extents[ORC_MAX_RANK];
  int64_t src_strides[ORC_MAX_RANK];
  int64_t dst_strides[ORC_MAX_RANK];
  int64_t pad_lo[ORC_MAX_RANK];
  int64_t pad_hi[ORC_MAX_RANK];
  int32_t src_width; /* bytes per source element */
  int32_t dst_width; /* bytes per destination element */
  int32_t has_fill;
  uint64_t fill_bits;
  int32_t result_rank;
  int64_t result_extents[ORC_MAX_RANK];
  int32_t nsymbols;
  int64_t symbols[ORC_MAX_SYMBOLS];
  int32_t nstages;
  orc_stage stages[ORC_MAX_STAGES];
} orc_program;

/* Execute the whole program: dst receives the dense padded result.
 * Returns 0, or 1 with a message (channel out of range, bad expression). */
int orc_execute(const orc_program *p, const void *src, void *dst, char *err,
                size_t cap);

/* Execute the physical outer-row window [row_begin, row_end) of the padded
 * result (axis 0 of the coalesced layout, pad rows included). dst receives the
 * window only; channels keep their global result coordinates. */
int orc_execute_rows(const orc_program *p, const void *src, void *dst,
                     int64_t row_begin, int64_t row_end, char *err, size_t cap);

/* Scalar contract, exposed for the witness-vector tests. */
uint16_t orc_narrow_f16(uint32_t f32_bits);
uint16_t orc_narrow_bf16(uint32_t f32_bits);
uint32_t orc_widen_f16(uint16_t h);
uint32_t orc_widen_bf16(uint16_t b);
int8_t orc_quantize(uint32_t f32_bits, float inv_scale);
uint32_t orc_dequantize(int8_t q, int32_t zero_point, float scale);
float orc_reciprocal(float scale);

#endif
