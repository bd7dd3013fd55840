/* sym_b200 -- thin C-ABI CUDA layer (libsb_cuda.so).
 *
 * The C++ host runtime (libsb_runtime.so) reaches the GPU only through these
 * functions: plain pointers, sizes and POD descriptors, streams and events
 * erased to void*, and int status codes (0 = success, otherwise a
 * cudaError_t value or one of the SBC_E* codes below). No CUDA or torch type
 * appears here, the convention of the reference's own CUDA headers
 * (libreloc/include/reloc/CudaKernels.h:3-9, CudaBackend.h:5-9).
 *
 * Replaces:
 *  - the reference's CudaBackend runtime calls: non-blocking streams,
 *    cudaHostAlloc staging, cudaMemcpyAsync, events, cross-stream waits,
 *    pointer-attribute checks (libreloc/cuda/CudaBackend.cu:55-282);
 *  - every transform kernel of libreloc/cuda/CudaKernels.cu (launchers at
 *    libreloc/include/reloc/CudaKernels.h:25-122) by four fused families
 *    that take the whole bound layout plus the value-stage chain:
 *      sbc_relocate_generic    any rank <= 8 layout, pads, any channel map;
 *      sbc_relocate_contiguous rank-1 unit-stride runs (quantize/dequantize/casts);
 *      sbc_relocate_runs       outer-axis permutations moving whole unit-stride
 *                              rows ([B,S,H,D] -> [B,H,S,D]);
 *      sbc_relocate_transpose  (batched) 2-D transposes with pads, tiled in
 *                              shared memory (f32 transpose, NCHW->NHWC+pad+f16,
 *                              int8 [out,in] -> f16 [in,out] dequant).
 */
#ifndef SYM_B200_SB_CUDA_H
#define SYM_B200_SB_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SBC_MAX_RANK 8
#define SBC_MAX_STAGES 4
#define SBC_MAX_TOKENS 16
#define SBC_MAX_SYMBOLS 8

/* Status codes beyond cudaError_t (kept far from its range). */
#define SBC_EINVAL 10001      /* descriptor violates the launcher's preconditions */
#define SBC_EUNSUPPORTED 10002 /* layout not of this kernel family */

enum sbc_stage_op {
  SBC_NARROW_F16 = 0,  /* cast f32 -> f16, ieee_rne */
  SBC_NARROW_BF16 = 1, /* cast f32 -> bf16, ieee_rne */
  SBC_WIDEN_F16 = 2,   /* cast f16 -> f32, exact */
  SBC_WIDEN_BF16 = 3,  /* cast bf16 -> f32, exact */
  SBC_QUANTIZE = 4,    /* f32 -> s8, symmetric_rne (param = reciprocal scales) */
  SBC_DEQUANTIZE = 5   /* s8 -> f32, affine (param = declared scales) */
};

enum sbc_channel_kind {
  SBC_CH_NONE = 0,   /* one parameter for every element */
  SBC_CH_AXIS = 1,   /* channel = (padded coordinate of axis ch_axis / ch_div) % ch_mod */
  SBC_CH_OFFSET = 2, /* channel = result coordinate ch_dim decoded from the dst offset */
  SBC_CH_EXPR = 3    /* channel = postfix expression over result coordinates */
};

typedef struct {
  int32_t op;        /* sbc_stage_op */
  int32_t channel;   /* sbc_channel_kind */
  int32_t ch_axis;   /* SBC_CH_AXIS */
  int32_t ch_dim;    /* SBC_CH_OFFSET */
  int64_t ch_div;    /* SBC_CH_AXIS, >= 1 */
  int64_t ch_mod;    /* SBC_CH_AXIS, 0 = no modulus */
  int64_t channel_length;
  const float *param;        /* device array: reciprocals (quantize) or scales (dequantize) */
  const int32_t *zero_point; /* device array or NULL */
  int32_t zp_mode;           /* 0 absent, 1 broadcast zero_point[0], 2 per channel */
  int32_t ntokens;
  int32_t token_op[SBC_MAX_TOKENS];
  int64_t token_value[SBC_MAX_TOKENS];
} sbc_stage;

/* One launch: produce the destination elements whose PADDED coordinates lie
 * in the box [box_lo, box_hi) of the coalesced layout. A coordinate c of axis
 * k is valid when pad_lo[k] <= c < pad_lo[k] + extents[k]; its source
 * coordinate is c - pad_lo[k]. Valid cells read
 *   src[sum((c_k - pad_lo_k) * src_strides_k) - src_offset]
 * through the stage chain; cells outside the valid box get fill_bits. Both go
 * to dst[sum(c_k * dst_strides_k) - dst_offset]. */
typedef struct {
  int32_t rank;
  int32_t src_width; /* bytes per source element: 1, 2, 4 or 8 */
  int32_t dst_width; /* bytes per destination element */
  int32_t has_fill;
  uint64_t fill_bits;
  int64_t extents[SBC_MAX_RANK];
  int64_t src_strides[SBC_MAX_RANK];
  int64_t dst_strides[SBC_MAX_RANK];
  int64_t pad_lo[SBC_MAX_RANK];
  int64_t box_lo[SBC_MAX_RANK];
  int64_t box_hi[SBC_MAX_RANK];
  const void *src; /* device pointer (HBM) or mapped pinned host memory */
  void *dst;       /* device pointer */
  /* Device word (or NULL) that a kernel sets to 1 when a channel index falls
   * outside its parameter table; such elements are skipped, never read past
   * the table. The runtime reports it as channel_out_of_range. */
  int32_t *status;
  /* Word (or NULL) that a kernel with bounded waits sets to 2 when a wait
   * runs out (a TMA copy it waited for never landed; the kernel left early
   * and its output is incomplete). Device memory or mapped pinned host
   * memory; the caller clears it and reads it after the launch completed. */
  int32_t *fault;
  int64_t src_offset;
  int64_t dst_offset;
  int32_t result_rank;
  int32_t nsymbols;
  int64_t result_strides[SBC_MAX_RANK];
  int64_t result_extents[SBC_MAX_RANK];
  int64_t symbols[SBC_MAX_SYMBOLS];
  int32_t nstages;
  int32_t reserved;
  sbc_stage stages[SBC_MAX_STAGES];
} sbc_relocate;

/* ---- kernels (asynchronous on `stream`; NULL = the legacy default stream) */
int sbc_relocate_generic(const sbc_relocate *desc, void *stream);
int sbc_relocate_contiguous(const sbc_relocate *desc, void *stream);
/* Rank >= 2 layouts whose last axis is unit-stride on both sides (outer axes
 * permuted, outer pads, one parameter per tensor or per run);
 * SBC_EUNSUPPORTED when the descriptor does not fit. */
int sbc_relocate_runs(const sbc_relocate *desc, void *stream);
int sbc_relocate_transpose(const sbc_relocate *desc, void *stream);
/* One TMA tile launch over `n` (<= 8) separately stored blocks of source
 * rows: `srcs[j]` holds the rows [row_bounds[j], row_bounds[j+1]) of axis 1
 * (the source-row axis of a rank-2 transpose; device memory, this GPU's or a
 * peer's), which together are the box's whole axis-1 range. `desc->src` is
 * not read. SBC_EUNSUPPORTED when the box or a block does not fit the tile
 * kernel (each block a multiple of 64 rows, TMA-aligned); the caller then
 * launches per block. */
int sbc_relocate_transpose_shards(const sbc_relocate *desc, const void *const *srcs, const int64_t *row_bounds,
                                  int32_t n, void *stream);
/* dst[i] = low `width` bytes of `bits`, i in [0, count). */
int sbc_fill(void *dst, int64_t count, int32_t width, uint64_t bits, void *stream);
/* Kernels launched by this library since load (instrumentation). */
uint64_t sbc_launch_count(void);
/* Launches since load of kernels with bounded waits, the only kernels that
 * write a descriptor's `fault` word: while it has not moved, no fault word
 * can have been set. */
uint64_t sbc_wait_launch_count(void);
/* Time limit of every bounded wait inside the kernels launched from now on
 * (nanoseconds of the GPU's global timer; 0 restores the default, one
 * second). */
void sbc_set_wait_limit_ns(uint64_t ns);

/* ---- test hooks (never armed by the library itself) ---------------------
 * Failure injection for the tests of the error paths; neither hook faults,
 * traps or hangs a GPU.
 *
 * sbc_test_fault_mode: make this layer's CUDA calls report cudaErrorUnknown
 * on the host without issuing them (the work already queued still runs):
 *   0 off;
 *   1 every event record fails;
 *   2 event records and stream synchronizations fail (completion unknown);
 *   3 the third host-to-device copy after arming fails;
 *   4 as 3, and stream synchronizations fail (completion unknown);
 *   5 event synchronizations fail;
 *   6 event and stream synchronizations fail (completion unknown).
 *
 * sbc_test_withhold_tile: the next TMA tile launch (any device) issues no
 * copy and no arrival for its job `job`, so the warps that wait for that
 * tile run out of their bounded wait after `wait_limit_ns` (0: the current
 * limit), set the descriptor's fault word and leave; the launch after it is
 * normal again. job = UINT32_MAX disarms. */
int sbc_test_fault_mode(int mode);
void sbc_test_withhold_tile(uint32_t job, uint64_t wait_limit_ns);

/* ---- devices, memory and copies */
int sbc_device_count(int *count);
int sbc_set_device(int device);
int sbc_get_device(int *device);
/* major/minor compute capability, SM count, global memory bytes. */
int sbc_device_info(int device, int *major, int *minor, int *sms, size_t *hbm_bytes);
int sbc_malloc_device(void **ptr, size_t bytes);
int sbc_free_device(void *ptr);
/* Pinned host memory; `mapped` != 0 also maps it into the device address space. */
int sbc_malloc_host(void **ptr, size_t bytes, int mapped);
int sbc_free_host(void *ptr);
int sbc_host_register(void *ptr, size_t bytes, int mapped);
int sbc_host_unregister(void *ptr);
/* Device address of mapped pinned host memory. */
int sbc_host_device_pointer(void *host, void **device);
/* CUDA IPC: the 64-byte handle of the device allocation that contains
 * `device_ptr` and the pointer's offset in it; the mapping of a peer
 * process's handle into this process (the allocation's base; peer access
 * enabled on first use); close unmaps. */
int sbc_ipc_get_handle(void *device_ptr, unsigned char handle[64], size_t *offset);
int sbc_ipc_open_handle(const unsigned char handle[64], void **device_ptr);
int sbc_ipc_close_handle(void *device_ptr);
/* Where a pointer lives: *kind 0 unregistered host, 1 pinned host, 2 device,
 * 3 managed; *device the owning ordinal (-1 for host). */
int sbc_pointer_info(const void *ptr, int *kind, int *device);
int sbc_memcpy_h2d_async(void *dst, const void *src, size_t bytes, void *stream);
int sbc_memcpy_d2h_async(void *dst, const void *src, size_t bytes, void *stream);
int sbc_memcpy_d2d_async(void *dst, const void *src, size_t bytes, void *stream);
/* Strided rows: `rows` copies of `width` bytes, pitches in bytes. */
int sbc_memcpy_h2d_2d_async(void *dst, size_t dpitch, const void *src, size_t spitch, size_t width, size_t rows,
                            void *stream);

/* ---- streams and events */
int sbc_stream_create(void **stream); /* non-blocking stream on the current device */
int sbc_stream_destroy(void *stream);
int sbc_stream_synchronize(void *stream);
int sbc_event_create(void **event, int timing);
int sbc_event_destroy(void *event);
int sbc_event_record(void *event, void *stream);
/* 0 complete, 1 not ready, otherwise an error. */
int sbc_event_query(void *event);
int sbc_event_synchronize(void *event);
int sbc_stream_wait_event(void *stream, void *event);
int sbc_event_elapsed_ms(void *start, void *stop, float *ms);
/* Most recent error string for a status code. */
const char *sbc_error_string(int status);

#ifdef __cplusplus
}
#endif

#endif
