// sym_b200 -- fused relocation kernels for sm_100a.
//
// Every kernel here performs the whole typed plan in one pass over HBM (or
// over mapped pinned host memory on the zero-copy route): index remap with
// pads, then the value-stage chain, then the store in the result layout. The
// element arithmetic is libreloc's C1 contract
// (docs/reloc-typed-semantics.md §3; reference kernels
// libreloc/cuda/CudaKernels.cu:149-238):
//   quantize   t = x * inv (one rounding), maxNum(t,-128), minNum(.,127), RNE
//   dequantize (q - zp) exactly, then one multiply
//   f32->f16 / f32->bf16 RNE narrowing, f16/bf16->f32 exact widening
// Multiplies use __fmul_rn so no FMA contraction can arise; the build passes
// neither --use_fast_math nor flush-to-zero. NaN inputs to the narrowing casts
// produce the reference's CPU NaN encoding (quiet bit + top payload bits), so
// outputs are bit-identical to the reference CPU executor for every input.
#include "sb_cuda.h"

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <cstdint>
#include <cstdlib>
#include <mutex>

namespace {

std::atomic<uint64_t> g_launches{0};
// Launches of kernels with bounded waits (the only writers of a descriptor's
// fault word): callers read their fault word only after one of these ran.
std::atomic<uint64_t> g_wait_launches{0};
// Time limit of each bounded wait (sbc_set_wait_limit_ns) and the test
// hook's withheld job with its own limit (sbc_test_withhold_tile).
constexpr uint64_t kDefaultWaitLimitNs = 1000000000ull; // one second
std::atomic<uint64_t> g_wait_ns{kDefaultWaitLimitNs};
std::atomic<uint32_t> g_withhold_job{UINT32_MAX};
std::atomic<uint64_t> g_withhold_ns{0};

// ---------------------------------------------------------------------------
// Scalar stage arithmetic
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint32_t narrow_f16(uint32_t x) {
  const uint32_t a = x & 0x7fffffffu;
  if (a > 0x7f800000u)
    return ((x >> 16) & 0x8000u) | 0x7e00u | ((a >> 13) & 0x3ffu);
  return __half_as_ushort(__float2half_rn(__uint_as_float(x)));
}

__device__ __forceinline__ uint32_t narrow_bf16(uint32_t x) {
  if ((x & 0x7fffffffu) > 0x7f800000u)
    return (x >> 16) | 0x40u;
  return __bfloat16_as_ushort(__float2bfloat16_rn(__uint_as_float(x)));
}

__device__ __forceinline__ uint32_t widen_f16(uint32_t h) {
  if ((h & 0x7c00u) == 0x7c00u && (h & 0x3ffu)) // NaN: payload shifted up
    return ((h & 0x8000u) << 16) | 0x7f800000u | ((h & 0x3ffu) << 13);
  return __float_as_uint(__half2float(__ushort_as_half(static_cast<unsigned short>(h))));
}

__device__ __forceinline__ uint32_t widen_bf16(uint32_t b) { return b << 16; }

__device__ __forceinline__ uint32_t quantize(uint32_t x, float inv) {
  float t = __fmul_rn(__uint_as_float(x), inv);
  t = fmaxf(t, -128.0f); // maxNum: NaN -> -128
  t = fminf(t, 127.0f);
  return static_cast<uint32_t>(__float2int_rn(t)) & 0xffu;
}

__device__ __forceinline__ uint32_t dequantize(uint32_t q, int32_t zp, float scale) {
  const int32_t d = static_cast<int32_t>(static_cast<int8_t>(q & 0xffu)) - zp;
  return __float_as_uint(__fmul_rn(static_cast<float>(d), scale));
}

// ---------------------------------------------------------------------------
// Stage chains. Common chains are specialized at compile time; CH_ANY
// interprets the descriptor's stage list.
// ---------------------------------------------------------------------------

enum Chain : int {
  CH_COPY = 0,
  CH_Q = 1,
  CH_DQ = 2,
  CH_F16 = 3,
  CH_BF16 = 4,
  CH_W16 = 5,
  CH_WB16 = 6,
  CH_DQ_F16 = 7,
  CH_DQ_BF16 = 8,
  CH_ANY = 9
};

__device__ __forceinline__ int32_t zp_of(const sbc_stage &s, int64_t c) {
  return s.zp_mode == 0 ? 0 : (s.zp_mode == 1 ? s.zero_point[0] : s.zero_point[c]);
}

__device__ __forceinline__ uint32_t apply_one(const sbc_stage &s, uint32_t v, int64_t c) {
  switch (s.op) {
  case SBC_NARROW_F16: return narrow_f16(v);
  case SBC_NARROW_BF16: return narrow_bf16(v);
  case SBC_WIDEN_F16: return widen_f16(v);
  case SBC_WIDEN_BF16: return widen_bf16(v);
  case SBC_QUANTIZE: return quantize(v, s.param[c]);
  default: return dequantize(v, zp_of(s, c), s.param[c]);
  }
}

/// Channel of stage `s` from the padded coordinates (AXIS kind) or the
/// global destination offset (OFFSET / EXPR kinds). Returns -1 when out of
/// range (the caller records the error and skips the element).
template <int R>
__device__ __forceinline__ int64_t channel_of(const sbc_relocate &d, const sbc_stage &s, const int64_t *coords,
                                              int64_t dglobal) {
  int64_t c = 0;
  if (s.channel == SBC_CH_NONE)
    return 0;
  if (s.channel == SBC_CH_AXIS) {
    c = coords[s.ch_axis] / s.ch_div;
    if (s.ch_mod)
      c %= s.ch_mod;
  } else if (s.channel == SBC_CH_OFFSET) {
    c = (dglobal / d.result_strides[s.ch_dim]) % d.result_extents[s.ch_dim];
  } else {
    int64_t rc[SBC_MAX_RANK];
    int64_t rest = dglobal;
    for (int j = 0; j < d.result_rank; ++j) {
      rc[j] = rest / d.result_strides[j];
      rest -= rc[j] * d.result_strides[j];
    }
    int64_t st[SBC_MAX_TOKENS];
    int sp = 0;
    for (int i = 0; i < s.ntokens; ++i) {
      const int op = s.token_op[i];
      const int64_t v = s.token_value[i];
      if (op == 0) st[sp++] = d.symbols[v];
      else if (op == 1) st[sp++] = v;
      else if (op == 7) st[sp++] = rc[v];
      else {
        const int64_t r = st[--sp], l = st[--sp];
        int64_t o = 0;
        if (op == 2) o = l + r;
        else if (op == 3) o = l - r;
        else if (op == 4) o = l * r;
        else {
          if (r == 0)
            return -1;
          int64_t q = l / r;
          if ((l % r != 0) && ((l < 0) != (r < 0)))
            --q;
          o = op == 5 ? q : l - q * r;
        }
        st[sp++] = o;
      }
    }
    c = sp == 1 ? st[0] : -1;
  }
  return (c < 0 || c >= s.channel_length) ? -1 : c;
}

/// Run the stage chain on one value. Returns false on a channel error.
template <int CHAIN, int R>
__device__ __forceinline__ bool run_chain(const sbc_relocate &d, uint32_t &v, const int64_t *coords, int64_t dglobal) {
  if constexpr (CHAIN == CH_COPY) {
    return true;
  } else if constexpr (CHAIN == CH_F16) {
    v = narrow_f16(v);
    return true;
  } else if constexpr (CHAIN == CH_BF16) {
    v = narrow_bf16(v);
    return true;
  } else if constexpr (CHAIN == CH_W16) {
    v = widen_f16(v);
    return true;
  } else if constexpr (CHAIN == CH_WB16) {
    v = widen_bf16(v);
    return true;
  } else if constexpr (CHAIN == CH_Q || CHAIN == CH_DQ || CHAIN == CH_DQ_F16 || CHAIN == CH_DQ_BF16) {
    const sbc_stage &s = d.stages[0];
    const int64_t c = channel_of<R>(d, s, coords, dglobal);
    if (c < 0)
      return false;
    if constexpr (CHAIN == CH_Q) {
      v = quantize(v, s.param[c]);
    } else {
      v = dequantize(v, zp_of(s, c), s.param[c]);
      if constexpr (CHAIN == CH_DQ_F16)
        v = narrow_f16(v);
      if constexpr (CHAIN == CH_DQ_BF16)
        v = narrow_bf16(v);
    }
    return true;
  } else {
    for (int k = 0; k < d.nstages; ++k) {
      const sbc_stage &s = d.stages[k];
      const int64_t c = channel_of<R>(d, s, coords, dglobal);
      if (c < 0)
        return false;
      v = apply_one(s, v, c);
    }
    return true;
  }
}

template <int W> struct Word;
template <> struct Word<1> { using T = uint8_t; };
template <> struct Word<2> { using T = uint16_t; };
template <> struct Word<4> { using T = uint32_t; };
template <> struct Word<8> { using T = unsigned long long; };

__device__ __forceinline__ void flag(const sbc_relocate &d) {
  if (d.status)
    atomicExch(d.status, 1);
}

// ---------------------------------------------------------------------------
// Generic gather over the destination box: any rank, pads, any channel map.
// ---------------------------------------------------------------------------

template <int WS, int WD, int CHAIN>
__global__ void __launch_bounds__(256) k_generic(const __grid_constant__ sbc_relocate d, int64_t total) {
  using S = typename Word<WS>::T;
  using D = typename Word<WD>::T;
  const S *src = static_cast<const S *>(d.src);
  D *dst = static_cast<D *>(d.dst);
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    int64_t coords[SBC_MAX_RANK];
    int64_t rem = i, so = 0, dg = 0;
    bool valid = true;
#pragma unroll
    for (int kk = 0; kk < SBC_MAX_RANK; ++kk) {
      const int k = SBC_MAX_RANK - 1 - kk;
      if (k >= d.rank)
        continue;
      const int64_t e = d.box_hi[k] - d.box_lo[k];
      const int64_t q = rem / e;
      const int64_t c = d.box_lo[k] + (rem - q * e);
      rem = q;
      coords[k] = c;
      dg += c * d.dst_strides[k];
      const int64_t v = c - d.pad_lo[k];
      if (v < 0 || v >= d.extents[k])
        valid = false;
      else
        so += v * d.src_strides[k];
    }
    if (!valid) {
      dst[dg - d.dst_offset] = static_cast<D>(d.fill_bits);
      continue;
    }
    if constexpr (WS == 8) {
      dst[dg - d.dst_offset] = static_cast<D>(src[so - d.src_offset]);
    } else {
      uint32_t v = static_cast<uint32_t>(src[so - d.src_offset]);
      if (!run_chain<CHAIN, SBC_MAX_RANK>(d, v, coords, dg)) {
        flag(d);
        continue;
      }
      dst[dg - d.dst_offset] = static_cast<D>(v);
    }
  }
}

// ---------------------------------------------------------------------------
// Contiguous runs: rank 1, unit strides, on the valid 16-byte aligned body
// (scalar head/tail and pad cells go to the generic kernel).
//
// Work is cut into units of U = 16 / max(WS, WD) elements: one 16-byte vector
// on the wider side and 16 / R bytes on the narrower one (R = wider / narrower
// width). A warp takes 32 * R consecutive units and lane l handles units
// k * 32 + l (k < R), so every load and every store instruction of the warp
// covers one contiguous span (512 bytes on the wide side): each instruction
// is fully coalesced, and a thread keeps R independent loads in flight.
// ---------------------------------------------------------------------------

template <int BYTES> struct Bytes;
template <> struct Bytes<4> { using T = uint32_t; };
template <> struct Bytes<8> { using T = uint2; };
template <> struct Bytes<16> { using T = uint4; };

/// Cells of a rank-1 box outside k_contiguous's aligned body: `nhead`
/// padded coordinates from `head_lo` and `ntail` from `tail_lo`.
struct ScalarEnds {
  int64_t head_lo = 0, tail_lo = 0;
  int32_t nhead = 0, ntail = 0;
};

template <int WS, int WD>
struct Units {
  static constexpr int MAXW = WS > WD ? WS : WD;
  static constexpr int MINW = WS < WD ? WS : WD;
  static constexpr int R = MAXW / MINW; // units per lane per warp block
  static constexpr int U = 16 / MAXW;   // elements per unit
};

template <int WS, int WD, int CHAIN, bool ENDS>
__global__ void __launch_bounds__(256) k_contiguous(const __grid_constant__ sbc_relocate d, int64_t vbegin,
                                                     int64_t nunits, ScalarEnds ends) {
  using S = typename Word<WS>::T;
  using D = typename Word<WD>::T;
  constexpr int R = Units<WS, WD>::R, U = Units<WS, WD>::U;
  using SU = typename Bytes<U * WS>::T;
  using DU = typename Bytes<U * WD>::T;
  const int64_t lo = d.pad_lo[0];
  // body start (16-byte aligned on both sides), viewed as arrays of units
  const SU *src = reinterpret_cast<const SU *>(static_cast<const S *>(d.src) + (vbegin - lo - d.src_offset));
  DU *dst = reinterpret_cast<DU *>(static_cast<D *>(d.dst) + (vbegin - d.dst_offset));
  // One parameter for every element (per-tensor scale): read it once per
  // thread instead of resolving a channel per element.
  constexpr bool kParam = CHAIN == CH_Q || CHAIN == CH_DQ || CHAIN == CH_DQ_F16 || CHAIN == CH_DQ_BF16;
  const bool uniform = kParam && d.stages[0].channel == SBC_CH_NONE && d.stages[0].channel_length >= 1;
  float p0 = 0.0f;
  int32_t zp0 = 0;
  if (uniform) {
    p0 = d.stages[0].param[0];
    zp0 = zp_of(d.stages[0], 0);
  }
  if (ENDS && blockIdx.x == 0) {
    // the unaligned head and tail cells (and pad cells there), one per thread
    for (int i = threadIdx.x; i < ends.nhead + ends.ntail; i += blockDim.x) {
      int64_t c = i < ends.nhead ? ends.head_lo + i : ends.tail_lo + (i - ends.nhead);
      const int64_t v = c - lo;
      D out;
      if (v < 0 || v >= d.extents[0]) {
        out = static_cast<D>(d.fill_bits);
      } else {
        uint32_t x = static_cast<uint32_t>(static_cast<const S *>(d.src)[v - d.src_offset]);
        if (!run_chain<CHAIN, 1>(d, x, &c, c)) {
          flag(d);
          continue;
        }
        out = static_cast<D>(x);
      }
      static_cast<D *>(d.dst)[c - d.dst_offset] = out;
    }
  }
  const int lane = threadIdx.x & 31;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  for (int64_t w = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5; w * 32 * R < nunits;
       w += nwarps) {
    union {
      SU q;
      S e[U];
    } in[R];
#pragma unroll
    for (int k = 0; k < R; ++k) {
      const int64_t u = (w * R + k) * 32 + lane;
      if (u < nunits)
        in[k].q = __ldcs(src + u); // streamed once: evict-first
    }
#pragma unroll
    for (int k = 0; k < R; ++k) {
      const int64_t u = (w * R + k) * 32 + lane;
      if (u >= nunits)
        continue;
      union {
        DU q;
        D e[U];
      } out;
      bool ok = true;
      if (uniform) {
#pragma unroll
        for (int i = 0; i < U; ++i) {
          uint32_t v = static_cast<uint32_t>(in[k].e[i]);
          if constexpr (CHAIN == CH_Q) {
            v = quantize(v, p0);
          } else if constexpr (kParam) {
            v = dequantize(v, zp0, p0);
            if constexpr (CHAIN == CH_DQ_F16)
              v = narrow_f16(v);
            if constexpr (CHAIN == CH_DQ_BF16)
              v = narrow_bf16(v);
          }
          out.e[i] = static_cast<D>(v);
        }
      } else {
#pragma unroll
        for (int i = 0; i < U; ++i) {
          int64_t c = vbegin + u * U + i; // padded coordinate
          uint32_t v = static_cast<uint32_t>(in[k].e[i]);
          ok &= run_chain<CHAIN, 1>(d, v, &c, c);
          out.e[i] = static_cast<D>(v);
        }
      }
      if (!ok) {
        flag(d);
        continue;
      }
      __stcs(dst + u, out.q);
    }
  }
}

// ---------------------------------------------------------------------------
// Narrow transposes: the destination-contiguous axis B has NB (2..4) padded
// cells and the destination is dense over (A, B) -- NCHW -> NHWC with three
// channels padded to four is the case. Each thread takes VA = 16 / WS
// consecutive cells of the source-contiguous axis A, reads one 16-byte vector
// from each of the NB source planes (valid B cells; pad cells take the fill),
// and writes its VA x NB destination cells as one contiguous run. A warp
// reads 512 contiguous bytes per plane and writes 32 * VA * NB * WD
// contiguous bytes: both sides coalesce without shared memory.
// Parameter stages are supported only with one parameter for every element.
// ---------------------------------------------------------------------------

/// Division by a runtime divisor d for numerators below 2^31:
/// n / d == (n * m) >> s with s = 31 + ceil(log2 d), m = ceil(2^s / d)
/// (exact because n * (m * d - 2^s) < 2^31 * d <= 2^s).
struct FastDiv {
  unsigned long long m;
  uint32_t s, d;
};

__device__ __forceinline__ uint32_t fdiv(uint32_t n, const FastDiv &f) {
  return static_cast<uint32_t>((static_cast<unsigned long long>(n) * f.m) >> f.s);
}

template <int BYTES> struct StoreVec { using T = uint4; };
template <> struct StoreVec<8> { using T = uint2; };
template <> struct StoreVec<4> { using T = uint32_t; };

/// Two f32 bit patterns narrowed to f16 (RNE) with one packed conversion,
/// x0 in the low half; NaNs keep narrow_f16's payload rule.
__device__ __forceinline__ uint32_t narrow2_f16(uint32_t x0, uint32_t x1) {
  if (max(x0 & 0x7fffffffu, x1 & 0x7fffffffu) > 0x7f800000u)
    return narrow_f16(x0) | (narrow_f16(x1) << 16);
  const __half2 h = __floats2half2_rn(__uint_as_float(x0), __uint_as_float(x1));
  return static_cast<uint32_t>(__half_as_ushort(__low2half(h))) |
         (static_cast<uint32_t>(__half_as_ushort(__high2half(h))) << 16);
}

/// One k_narrow item: VA source cells of axis A from each of the NB planes
/// (16-byte loads already issued into `in`; pad planes take the fill),
/// converted and stored as one contiguous run of VA x NB cells at `dp`.
template <int WS, int WD, int CHAIN, int NB>
__device__ __forceinline__ void narrow_item(const uint4 (&in)[NB], const bool (&valid)[NB], uint8_t *dp,
                                            uint32_t fill, float p0, int32_t zp0) {
  using S = typename Word<WS>::T;
  using D = typename Word<WD>::T;
  constexpr int VA = 16 / WS;
  constexpr int RUN = VA * NB * WD;
  constexpr int SV = RUN % 16 == 0 ? 16 : RUN % 8 == 0 ? 8 : 4;
  using ST = typename StoreVec<SV>::T;
  union {
    ST q[RUN / SV];
    D e[VA * NB];
    uint32_t w[(RUN + 3) / 4];
  } out;
  if constexpr (CHAIN == CH_F16 && WS == 4 && WD == 2 && NB % 2 == 0) {
    // channel pairs (j, j + 1) of one cell: one packed conversion
#pragma unroll
    for (int j = 0; j < NB; j += 2) {
      const uint4 x = in[j], y = in[j + 1];
      const uint32_t xs[4] = {x.x, x.y, x.z, x.w}, ys[4] = {y.x, y.y, y.z, y.w};
#pragma unroll
      for (int i = 0; i < VA; ++i) {
        uint32_t w;
        if (valid[j] && valid[j + 1])
          w = narrow2_f16(xs[i], ys[i]);
        else if (valid[j])
          w = narrow_f16(xs[i]) | (fill << 16);
        else if (valid[j + 1])
          w = fill | (narrow_f16(ys[i]) << 16);
        else
          w = fill | (fill << 16);
        out.w[(i * NB + j) / 2] = w;
      }
    }
  } else {
#pragma unroll
    for (int j = 0; j < NB; ++j) {
      union {
        uint4 q;
        S e[VA];
      } v;
      v.q = in[j];
#pragma unroll
      for (int i = 0; i < VA; ++i) {
        uint32_t x = static_cast<uint32_t>(v.e[i]);
        if constexpr (CHAIN == CH_F16)
          x = narrow_f16(x);
        else if constexpr (CHAIN == CH_BF16)
          x = narrow_bf16(x);
        else if constexpr (CHAIN == CH_W16)
          x = widen_f16(x);
        else if constexpr (CHAIN == CH_WB16)
          x = widen_bf16(x);
        else if constexpr (CHAIN == CH_Q)
          x = quantize(x, p0);
        else if constexpr (CHAIN == CH_DQ)
          x = dequantize(x, zp0, p0);
        out.e[i * NB + j] = static_cast<D>(valid[j] ? x : fill);
      }
    }
  }
  ST *sp = reinterpret_cast<ST *>(dp);
#pragma unroll
  for (int i = 0; i < RUN / SV; ++i)
    __stcs(sp + i, out.q[i]);
}

/// V == 1: one item per thread (each resolves its own batch index). V > 1
/// (the host checks that a batch holds a whole number of 32 * V items): a
/// warp takes 32 * V consecutive items of one batch, resolves the batch and
/// the base offsets once, and lane l takes items l, l + 32, ..., issuing all
/// of its 16-byte loads before the first conversion.
template <int WS, int WD, int CHAIN, int NB, int V>
__global__ void __launch_bounds__(256) k_narrow(const __grid_constant__ sbc_relocate d, FastDiv per_batch,
                                                 uint32_t total) {
  using S = typename Word<WS>::T;
  constexpr int VA = 16 / WS;
  const int ax_a = d.rank - 2, ax_b = d.rank - 1;
  const int64_t Sb = d.src_strides[ax_b];
  const int64_t lo_b = d.pad_lo[ax_b], hi_b = d.pad_lo[ax_b] + d.extents[ax_b];
  const int64_t b0 = d.box_lo[ax_b];
  const S *src = static_cast<const S *>(d.src);
  uint8_t *dst = static_cast<uint8_t *>(d.dst);
  const sbc_stage &s = d.stages[0];
  float p0 = 0.0f;
  int32_t zp0 = 0;
  if constexpr (CHAIN == CH_Q || CHAIN == CH_DQ) {
    p0 = s.param[0];
    zp0 = zp_of(s, 0);
  }
  const uint32_t fill = static_cast<uint32_t>(static_cast<typename Word<WD>::T>(d.fill_bits));
  bool valid[NB];
#pragma unroll
  for (int j = 0; j < NB; ++j)
    valid[j] = b0 + j >= lo_b && b0 + j < hi_b;
  // element offsets of item g's first source cell (plane b0) and destination cell
  auto bases = [&](uint32_t g, int64_t &sbase, int64_t &dbase) {
    const uint32_t n = d.rank == 3 ? fdiv(g, per_batch) : 0; // total < 2^31 (host-checked)
    const int64_t a = d.box_lo[ax_a] + static_cast<int64_t>(g - n * per_batch.d) * VA;
    sbase = (a - d.pad_lo[ax_a]) - d.src_offset + (b0 - lo_b) * Sb;
    dbase = a * NB + b0 - d.dst_offset; // dst_strides[ax_a] == NB (host-checked)
    if (d.rank == 3) {
      sbase += (d.box_lo[0] + n - d.pad_lo[0]) * d.src_strides[0];
      dbase += (d.box_lo[0] + n) * d.dst_strides[0];
    }
  };
  if constexpr (V == 1) {
    for (uint32_t g = blockIdx.x * blockDim.x + threadIdx.x; g < total; g += gridDim.x * blockDim.x) {
      int64_t sbase, dbase;
      bases(g, sbase, dbase);
      uint4 in[NB] = {};
#pragma unroll
      for (int j = 0; j < NB; ++j)
        if (valid[j])
          in[j] = __ldcs(reinterpret_cast<const uint4 *>(src + sbase + j * Sb));
      narrow_item<WS, WD, CHAIN, NB>(in, valid, dst + dbase * WD, fill, p0, zp0);
    }
  } else {
    const int lane = threadIdx.x & 31;
    const uint32_t nspans = total / (32 * V);
    const uint32_t warps = gridDim.x * (blockDim.x / 32);
    for (uint32_t sp = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5); sp < nspans; sp += warps) {
      int64_t sbase, dbase;
      bases(sp * (32 * V), sbase, dbase);
      uint4 in[V][NB] = {};
#pragma unroll
      for (int v = 0; v < V; ++v)
#pragma unroll
        for (int j = 0; j < NB; ++j)
          if (valid[j])
            in[v][j] = __ldcs(reinterpret_cast<const uint4 *>(src + sbase + j * Sb + (v * 32 + lane) * VA));
#pragma unroll
      for (int v = 0; v < V; ++v)
        narrow_item<WS, WD, CHAIN, NB>(in[v], valid, dst + (dbase + (v * 32 + lane) * VA * NB) * WD, fill, p0,
                                       zp0);
    }
  }
}

// ---------------------------------------------------------------------------
// Runs: the last axis is unit-stride in both the source and the destination,
// so each destination row of that axis is one contiguous run of the source
// (leading axes permuted: [B,S,H,D] -> [B,H,S,D], swaps of outer axes).
// The box is cut into units of U = 16 / max(WS, WD) elements of the last
// axis, taken in destination order. With V > 1 (rows a multiple of 32 * V
// units long) a warp takes a span of 32 * V consecutive units inside one
// row: it resolves the row's outer coordinates (one magic-number division
// per outer axis) and parameter once, then lane l moves units l, l + 32, ...
// so every load and store instruction of the warp is one contiguous span.
// With V == 1 each thread resolves its own unit's row. Rows inside an outer
// pad take the fill. Parameters: one per tensor, or one per run (a channel
// on an outer axis).
// ---------------------------------------------------------------------------

struct RunsGeom {
  FastDiv upr;                   // units per row of the last axis
  FastDiv ext[SBC_MAX_RANK - 1]; // box extents of the outer axes
};

/// Row `row` of the box's outer axes: source and destination element offsets
/// of its first cell, validity (false inside an outer pad) and the stage-0
/// parameter (and zero point) of the run. False return: channel out of range.
template <int CHAIN>
__device__ __forceinline__ bool runs_row(const sbc_relocate &d, const RunsGeom &g, uint32_t row, int64_t &so,
                                         int64_t &dg, bool &valid, float &p, int32_t &zp) {
  constexpr bool kParam = CHAIN == CH_Q || CHAIN == CH_DQ || CHAIN == CH_DQ_F16 || CHAIN == CH_DQ_BF16;
  const int last = d.rank - 1;
  int64_t coords[SBC_MAX_RANK - 1];
  so = 0;
  dg = 0;
  valid = true;
#pragma unroll
  for (int kk = 0; kk < SBC_MAX_RANK - 1; ++kk) {
    const int k = SBC_MAX_RANK - 2 - kk; // innermost outer axis first
    if (k >= last)
      continue;
    const uint32_t q = fdiv(row, g.ext[k]);
    const int64_t c = d.box_lo[k] + (row - q * g.ext[k].d);
    row = q;
    coords[k] = c;
    dg += c * d.dst_strides[k];
    const int64_t v = c - d.pad_lo[k];
    if (v < 0 || v >= d.extents[k])
      valid = false;
    else
      so += v * d.src_strides[k];
  }
  if constexpr (kParam) {
    const sbc_stage &s = d.stages[0];
    int64_t c = 0;
    if (s.channel == SBC_CH_AXIS) {
      c = coords[s.ch_axis] / s.ch_div;
      if (s.ch_mod)
        c %= s.ch_mod;
    }
    if (c >= s.channel_length)
      return false;
    p = s.param[c];
    zp = zp_of(s, c);
  }
  return true;
}

/// Convert one unit (U source cells) and store it at `dp`.
template <int WS, int WD, int CHAIN, typename SU, typename DU>
__device__ __forceinline__ void runs_unit(const SU &src, DU *dp, float p, int32_t zp) {
  using S = typename Word<WS>::T;
  using D = typename Word<WD>::T;
  constexpr int U = Units<WS, WD>::U;
  union {
    SU q;
    S e[U];
  } in;
  in.q = src;
  union {
    DU q;
    D e[U];
    uint32_t w[(U * WD + 3) / 4];
  } out;
  if constexpr (CHAIN == CH_F16 && WS == 4 && WD == 2) {
#pragma unroll
    for (int u = 0; u < U; u += 2)
      out.w[u / 2] = narrow2_f16(in.e[u], in.e[u + 1]);
  } else {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      uint32_t v = static_cast<uint32_t>(in.e[u]);
      if constexpr (CHAIN == CH_F16)
        v = narrow_f16(v);
      else if constexpr (CHAIN == CH_BF16)
        v = narrow_bf16(v);
      else if constexpr (CHAIN == CH_W16)
        v = widen_f16(v);
      else if constexpr (CHAIN == CH_WB16)
        v = widen_bf16(v);
      else if constexpr (CHAIN == CH_Q)
        v = quantize(v, p);
      else if constexpr (CHAIN == CH_DQ)
        v = dequantize(v, zp, p);
      else if constexpr (CHAIN == CH_DQ_F16)
        v = narrow_f16(dequantize(v, zp, p));
      else if constexpr (CHAIN == CH_DQ_BF16)
        v = narrow_bf16(dequantize(v, zp, p));
      out.e[u] = static_cast<D>(v);
    }
  }
  __stcs(dp, out.q);
}

template <int WS, int WD, int CHAIN, int V>
__global__ void __launch_bounds__(256) k_runs(const __grid_constant__ sbc_relocate d, const __grid_constant__ RunsGeom g,
                                               uint32_t nunits) {
  using S = typename Word<WS>::T;
  using D = typename Word<WD>::T;
  constexpr int U = Units<WS, WD>::U;
  using SU = typename Bytes<U * WS>::T;
  using DU = typename Bytes<U * WD>::T;
  const int last = d.rank - 1;
  const S *src = static_cast<const S *>(d.src) + (d.box_lo[last] - d.pad_lo[last] - d.src_offset);
  D *dst = static_cast<D *>(d.dst) + (d.box_lo[last] - d.dst_offset);
  if constexpr (V == 1) {
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < nunits; i += gridDim.x * blockDim.x) {
      const uint32_t row = fdiv(i, g.upr);
      const int64_t j = static_cast<int64_t>(i - row * g.upr.d) * U;
      int64_t so, dg;
      bool valid;
      float p = 0.0f;
      int32_t zp = 0;
      if (!runs_row<CHAIN>(d, g, row, so, dg, valid, p, zp)) {
        flag(d);
        continue;
      }
      DU *dp = reinterpret_cast<DU *>(dst + dg + j);
      if (!valid) {
        union {
          DU q;
          D e[U];
        } out;
#pragma unroll
        for (int u = 0; u < U; ++u)
          out.e[u] = static_cast<D>(d.fill_bits);
        __stcs(dp, out.q);
        continue;
      }
      runs_unit<WS, WD, CHAIN>(__ldcs(reinterpret_cast<const SU *>(src + so + j)), dp, p, zp);
    }
  } else {
    const int lane = threadIdx.x & 31;
    const uint32_t nspans = nunits / (32 * V); // host: rows are whole spans
    const uint32_t warps = gridDim.x * (blockDim.x / 32);
    for (uint32_t sp = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5); sp < nspans; sp += warps) {
      const uint32_t u0 = sp * (32 * V);
      const uint32_t row = fdiv(u0, g.upr);
      const int64_t j0 = static_cast<int64_t>(u0 - row * g.upr.d + lane) * U;
      int64_t so, dg;
      bool valid;
      float p = 0.0f;
      int32_t zp = 0;
      if (!runs_row<CHAIN>(d, g, row, so, dg, valid, p, zp)) {
        flag(d);
        continue;
      }
      DU *dp = reinterpret_cast<DU *>(dst + dg + j0);
      if (!valid) {
        union {
          DU q;
          D e[U];
        } out;
#pragma unroll
        for (int u = 0; u < U; ++u)
          out.e[u] = static_cast<D>(d.fill_bits);
#pragma unroll
        for (int v = 0; v < V; ++v)
          __stcs(dp + v * 32, out.q);
        continue;
      }
      const SU *sp_ = reinterpret_cast<const SU *>(src + so + j0);
      SU in[V];
#pragma unroll
      for (int v = 0; v < V; ++v)
        in[v] = __ldcs(sp_ + v * 32);
#pragma unroll
      for (int v = 0; v < V; ++v)
        runs_unit<WS, WD, CHAIN>(in[v], dp + v * 32, p, zp);
    }
  }
}

// ---------------------------------------------------------------------------
// Tiled transpose. Layout (rank 2): axis A (src stride 1) then axis B (dst
// stride 1); rank 3 adds a leading batch axis N. A tile of TA x TB padded
// coordinates is read along A (coalesced in the source), converted, staged in
// shared memory, and written along B (coalesced in the destination).
// ---------------------------------------------------------------------------

template <int WS, int WD, int CHAIN>
__global__ void __launch_bounds__(256) k_transpose(const __grid_constant__ sbc_relocate d, int ta, int tb,
                                                    int64_t tiles_a, int64_t tiles_b, int64_t nbatch) {
  using S = typename Word<WS>::T;
  using D = typename Word<WD>::T;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  D *tile = reinterpret_cast<D *>(smem_raw);
  const int pitch = tb + 1;
  const int r = d.rank;
  const int ax_a = r - 2, ax_b = r - 1;
  const S *src = static_cast<const S *>(d.src);
  D *dst = static_cast<D *>(d.dst);
  const int64_t tiles = tiles_a * tiles_b;
  for (int64_t job = blockIdx.x; job < tiles * nbatch; job += gridDim.x) {
    const int64_t n_idx = job / tiles;
    const int64_t t = job - n_idx * tiles;
    const int64_t ta_i = t % tiles_a, tb_i = t / tiles_a;
    int64_t coords[3];
    int64_t nsrc = 0, ndst = 0;
    bool nvalid = true;
    if (r == 3) {
      const int64_t cn = d.box_lo[0] + n_idx;
      coords[0] = cn;
      ndst = cn * d.dst_strides[0];
      const int64_t vn = cn - d.pad_lo[0];
      nvalid = vn >= 0 && vn < d.extents[0];
      nsrc = vn * d.src_strides[0];
    }
    const int64_t a0 = d.box_lo[ax_a] + ta_i * ta, b0 = d.box_lo[ax_b] + tb_i * tb;
    const int64_t a_end = min(a0 + ta, d.box_hi[ax_a]), b_end = min(b0 + tb, d.box_hi[ax_b]);
    const int na = static_cast<int>(a_end - a0), nb = static_cast<int>(b_end - b0);
    // load + convert: consecutive threads take consecutive A (source-contiguous)
    for (int e = threadIdx.x; e < na * nb; e += blockDim.x) {
      const int al = e % na, bl = e / na;
      const int64_t ca = a0 + al, cb = b0 + bl;
      const int64_t va = ca - d.pad_lo[ax_a], vb = cb - d.pad_lo[ax_b];
      D out;
      if (!nvalid || va < 0 || va >= d.extents[ax_a] || vb < 0 || vb >= d.extents[ax_b]) {
        out = static_cast<D>(d.fill_bits);
      } else {
        uint32_t v = static_cast<uint32_t>(src[nsrc + va + vb * d.src_strides[ax_b] - d.src_offset]);
        coords[ax_a] = ca;
        coords[ax_b] = cb;
        const int64_t dg = ndst + ca * d.dst_strides[ax_a] + cb;
        if (!run_chain<CHAIN, 3>(d, v, coords, dg)) {
          flag(d);
          v = 0;
        }
        out = static_cast<D>(v);
      }
      tile[al * pitch + bl] = out;
    }
    __syncthreads();
    // store: consecutive threads take consecutive B (destination-contiguous)
    for (int e = threadIdx.x; e < na * nb; e += blockDim.x) {
      const int al = e / nb, bl = e % nb;
      dst[ndst + (a0 + al) * d.dst_strides[ax_a] + b0 + bl - d.dst_offset] = tile[al * pitch + bl];
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// Vectorized tiled transpose for unpadded, 16-byte aligned (batched) 2-D
// transposes -- the hot kernel of the int8 weight fetch.
//
// A tile is 128 source bytes along A by 128 destination bytes along B
// (s8 -> f16: 128 x 64 elements). Load: each thread moves one 16-byte
// chunk of a source row into shared memory (8 threads per 128-byte row,
// fully coalesced). Shared rows are 128 bytes with the 16-byte chunk index
// XOR-swizzled by (row / VD) so that the transposed reads below hit eight
// distinct chunks per quarter-warp. Store: each thread gathers VD = 16/WD
// elements of one destination row from VD shared rows, runs the stage chain
// with the per-channel parameter of its coordinate, and writes one 16-byte
// chunk (8 threads per 128-byte destination row segment). Edge tiles take a
// guarded element path. CH_ON: 0 = no per-channel stage, 1 = channel is the
// A coordinate, 2 = channel is the B coordinate (divisor 1, no modulus).
// ---------------------------------------------------------------------------

template <int CHAIN>
__device__ __forceinline__ bool chain_at(const sbc_relocate &d, uint32_t &v, int64_t ch) {
  if constexpr (CHAIN == CH_COPY) {
    return true;
  } else if constexpr (CHAIN == CH_F16) {
    v = narrow_f16(v);
    return true;
  } else if constexpr (CHAIN == CH_BF16) {
    v = narrow_bf16(v);
    return true;
  } else if constexpr (CHAIN == CH_W16) {
    v = widen_f16(v);
    return true;
  } else if constexpr (CHAIN == CH_WB16) {
    v = widen_bf16(v);
    return true;
  } else if constexpr (CHAIN == CH_Q || CHAIN == CH_DQ || CHAIN == CH_DQ_F16 || CHAIN == CH_DQ_BF16) {
    const sbc_stage &s = d.stages[0];
    const int64_t c = s.channel == SBC_CH_NONE ? 0 : ch;
    if (c >= s.channel_length)
      return false;
    if constexpr (CHAIN == CH_Q) {
      v = quantize(v, s.param[c]);
    } else {
      v = dequantize(v, zp_of(s, c), s.param[c]);
      if constexpr (CHAIN == CH_DQ_F16)
        v = __half_as_ushort(__float2half_rn(__uint_as_float(v))); // finite: no NaN path
      if constexpr (CHAIN == CH_DQ_BF16)
        v = __bfloat16_as_ushort(__float2bfloat16_rn(__uint_as_float(v)));
    }
    return true;
  } else {
    for (int k = 0; k < d.nstages; ++k) {
      const sbc_stage &s = d.stages[k];
      const int64_t c = s.channel == SBC_CH_NONE ? 0 : ch;
      if (c >= s.channel_length)
        return false;
      v = apply_one(s, v, c);
    }
    return true;
  }
}

template <int W>
__device__ __forceinline__ uint32_t load_elem(const uint8_t *p) {
  if constexpr (W == 1)
    return *p;
  else if constexpr (W == 2)
    return *reinterpret_cast<const uint16_t *>(p);
  else
    return *reinterpret_cast<const uint32_t *>(p);
}

template <int WS, int WD, int CHAIN, int CH_ON>
__global__ void __launch_bounds__(256) k_tile(const __grid_constant__ sbc_relocate d, int64_t tiles_b,
                                              int64_t tiles, int64_t nbatch) {
  using D = typename Word<WD>::T;
  constexpr int TA = 128 / WS, TB = 128 / WD, VD = 16 / WD, VS = 16 / WS;
  __shared__ __align__(16) uint8_t sm[TB * 128];
  const int t = threadIdx.x;
  const int r = d.rank, ax_a = r - 2, ax_b = r - 1;
  const int64_t Sb = d.src_strides[ax_b], Da = d.dst_strides[ax_a];
  for (int64_t job = blockIdx.x; job < tiles * nbatch; job += gridDim.x) {
    const int64_t n_idx = job / tiles, tile = job - n_idx * tiles;
    const int64_t tb_i = tile % tiles_b, ta_i = tile / tiles_b;
    int64_t nsrc = 0, ndst = 0;
    if (r == 3) {
      const int64_t cn = d.box_lo[0] + n_idx;
      nsrc = cn * d.src_strides[0];
      ndst = cn * d.dst_strides[0];
    }
    const int64_t a0 = d.box_lo[ax_a] + ta_i * TA, b0 = d.box_lo[ax_b] + tb_i * TB;
    const int na = static_cast<int>(min(static_cast<int64_t>(TA), d.box_hi[ax_a] - a0));
    const int nb = static_cast<int>(min(static_cast<int64_t>(TB), d.box_hi[ax_b] - b0));
    const bool full = na == TA && nb == TB;
    const uint8_t *srcb = static_cast<const uint8_t *>(d.src) + (nsrc + a0 + b0 * Sb - d.src_offset) * WS;
    uint8_t *dstb = static_cast<uint8_t *>(d.dst) + (ndst + a0 * Da + b0 - d.dst_offset) * WD;
    // ---- load: 16-byte chunks of TB source rows
#pragma unroll
    for (int p = 0; p < TB / 32; ++p) {
      const int row = p * 32 + (t >> 3), c = t & 7;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (full) {
        v = __ldcs(reinterpret_cast<const uint4 *>(srcb + row * Sb * WS + c * 16));
      } else if (row < nb) {
        uint8_t *vb = reinterpret_cast<uint8_t *>(&v);
        for (int e = 0; e < VS; ++e)
          if (c * VS + e < na)
            for (int k = 0; k < WS; ++k)
              vb[e * WS + k] = srcb[row * Sb * WS + (c * VS + e) * WS + k];
      }
      *reinterpret_cast<uint4 *>(sm + row * 128 + ((c ^ ((row / VD) & 7)) << 4)) = v;
    }
    __syncthreads();
    // ---- store: one 16-byte destination chunk per thread per pass
    const int c = t & 7;
    // Quantize/dequantize parameters of this thread's VD columns, loaded once
    // per tile when the channel is the B coordinate.
    constexpr bool QDQ = CHAIN == CH_Q || CHAIN == CH_DQ || CHAIN == CH_DQ_F16 || CHAIN == CH_DQ_BF16;
    float pscale[VD];
    int32_t pzp[VD];
    bool pok = true;
    if constexpr (QDQ) {
      const sbc_stage &s = d.stages[0];
#pragma unroll
      for (int j = 0; j < VD; ++j) {
        int64_t ch = (CH_ON == 2 && c * VD + j < nb) ? b0 + c * VD + j : 0;
        if (ch >= s.channel_length) {
          pok = false;
          ch = 0;
        }
        pscale[j] = s.param[ch];
        pzp[j] = zp_of(s, ch);
      }
    }
#pragma unroll
    for (int p = 0; p < TA / 32; ++p) {
      const int arow = p * 32 + (t >> 3);
      if (arow < na) {
        union {
          uint4 q;
          D e[VD];
        } out;
        const int xb = arow * WS; // byte column in the shared rows
        bool ok = pok;
        if constexpr (QDQ && CH_ON == 1) {
          const sbc_stage &s = d.stages[0];
          int64_t ch = a0 + arow;
          if (ch >= s.channel_length) {
            ok = false;
            ch = 0;
          }
#pragma unroll
          for (int j = 0; j < VD; ++j) {
            pscale[j] = s.param[ch];
            pzp[j] = zp_of(s, ch);
          }
        }
#pragma unroll
        for (int j = 0; j < VD; ++j) {
          const int brow = c * VD + j;
          uint32_t v = load_elem<WS>(sm + brow * 128 + (((xb >> 4) ^ (c & 7)) << 4) + (xb & 15));
          if constexpr (CHAIN == CH_Q) {
            v = quantize(v, pscale[j]);
          } else if constexpr (CHAIN == CH_DQ) {
            v = dequantize(v, pzp[j], pscale[j]);
          } else if constexpr (CHAIN == CH_DQ_F16) {
            v = __half_as_ushort(__float2half_rn(__uint_as_float(dequantize(v, pzp[j], pscale[j]))));
          } else if constexpr (CHAIN == CH_DQ_BF16) {
            v = __bfloat16_as_ushort(__float2bfloat16_rn(__uint_as_float(dequantize(v, pzp[j], pscale[j]))));
          } else {
            const int64_t ch = CH_ON == 2 ? b0 + brow : (CH_ON == 1 ? a0 + arow : 0);
            ok &= chain_at<CHAIN>(d, v, ch);
          }
          out.e[j] = static_cast<D>(v);
        }
        if (!ok)
          flag(d);
        uint8_t *dp = dstb + static_cast<int64_t>(arow) * Da * WD + c * 16;
        if (full) {
          __stcs(reinterpret_cast<uint4 *>(dp), out.q);
        } else {
          for (int j = 0; j < VD; ++j)
            if (c * VD + j < nb)
              reinterpret_cast<D *>(dp)[j] = out.e[j];
        }
      }
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// int8-source tile transpose (dequantize -> f16/bf16/f32): the hot kernel.
//
// Same tile and swizzle as k_tile, but each thread owns a 4 x VD block of
// the output (4 destination rows A, VD = 16/WD destination columns B): it
// reads VD 32-bit shared words, each holding the 4 A-consecutive int8 values
// of one source row, so one shared load feeds 4 outputs. The block loops over
// tiles with the next tile's 16-byte global loads issued before the current
// tile's conversion and stores (register prefetch), keeping HBM reads in
// flight while the SM converts. Per-channel parameters along B are loaded once
// per tile.
// ---------------------------------------------------------------------------

template <int WD, int CHAIN, int CH_ON>
__global__ void __launch_bounds__(256, 4) k_tile_s8(const __grid_constant__ sbc_relocate d, FastDiv div_b,
                                                    FastDiv div_t, uint32_t total) {
  constexpr int TA = 128, TB = 128 / WD, VD = 16 / WD, LP = TB / 32;
  using D = typename Word<WD>::T;
  __shared__ __align__(16) uint8_t sm[TB * 128];
  const int t = threadIdx.x, ag = t >> 3, c = t & 7; // store block: rows 4*ag.., columns c*VD..
  const int r = d.rank, ax_a = r - 2, ax_b = r - 1;
  const int64_t Sb = d.src_strides[ax_b], Da = d.dst_strides[ax_a], DaB = Da * WD;
  const uint8_t *const src0 = static_cast<const uint8_t *>(d.src) - d.src_offset;
  uint8_t *const dst0 = static_cast<uint8_t *>(d.dst) - d.dst_offset * WD;
  const sbc_stage &s = d.stages[0];

  struct Tile {
    const uint8_t *src;
    uint8_t *dst;
    int64_t a0, b0;
    int na, nb;
  };
  auto tile_of = [&](uint32_t job) {
    Tile T;
    const uint32_t n_idx = fdiv(job, div_t), tile = job - n_idx * div_t.d;
    const uint32_t ta_i = fdiv(tile, div_b), tb_i = tile - ta_i * div_b.d;
    int64_t ns = 0, nd = 0;
    if (r == 3) {
      const int64_t cn = d.box_lo[0] + n_idx;
      ns = cn * d.src_strides[0];
      nd = cn * d.dst_strides[0];
    }
    T.a0 = d.box_lo[ax_a] + static_cast<int64_t>(ta_i) * TA;
    T.b0 = d.box_lo[ax_b] + static_cast<int64_t>(tb_i) * TB;
    T.na = static_cast<int>(min(static_cast<int64_t>(TA), d.box_hi[ax_a] - T.a0));
    T.nb = static_cast<int>(min(static_cast<int64_t>(TB), d.box_hi[ax_b] - T.b0));
    T.src = src0 + ns + T.a0 + T.b0 * Sb;
    T.dst = dst0 + (nd + T.a0 * Da + T.b0) * WD;
    return T;
  };
  auto load = [&](const Tile &T, uint4 (&v)[LP]) {
    const bool full = T.na == TA && T.nb == TB;
#pragma unroll
    for (int p = 0; p < LP; ++p) {
      const int row = p * 32 + (t >> 3);
      v[p] = make_uint4(0, 0, 0, 0);
      if (full) {
        v[p] = __ldcs(reinterpret_cast<const uint4 *>(T.src + row * Sb + c * 16));
      } else if (row < T.nb) {
        uint8_t *vb = reinterpret_cast<uint8_t *>(&v[p]);
        for (int e = 0; e < 16; ++e)
          if (c * 16 + e < T.na)
            vb[e] = T.src[row * Sb + c * 16 + e];
      }
    }
  };

  uint32_t job = blockIdx.x;
  uint4 pre[LP];
  if (job < total)
    load(tile_of(job), pre);
  for (; job < total; job += gridDim.x) {
    const Tile T = tile_of(job);
#pragma unroll
    for (int p = 0; p < LP; ++p) {
      const int row = p * 32 + (t >> 3);
      *reinterpret_cast<uint4 *>(sm + row * 128 + ((c ^ ((row / VD) & 7)) << 4)) = pre[p];
    }
    __syncthreads();
    if (job + gridDim.x < total)
      load(tile_of(job + gridDim.x), pre); // in flight during the conversion below

    // Parameters of this thread's VD columns. The int8 -> f32 conversion is
    // exact and uses the FP32 pipe: the biased byte (q + 128) is placed in
    // the mantissa of 2^23, and one subtraction of 2^23 + 128 + zp leaves the
    // integer q - zp exactly; one multiply by the scale follows (C1 affine).
    float ps[VD], bias[VD];
    bool ok = true;
#pragma unroll
    for (int j = 0; j < VD; ++j) {
      int64_t ch = 0;
      if constexpr (CH_ON == 2)
        ch = (c * VD + j < T.nb) ? T.b0 + c * VD + j : 0;
      if (ch >= s.channel_length) {
        ok = false;
        ch = 0;
      }
      ps[j] = s.param[ch];
      bias[j] = 8388736.0f + static_cast<float>(zp_of(s, ch));
    }
    uint32_t w[VD];
#pragma unroll
    for (int j = 0; j < VD; ++j) {
      const int row = c * VD + j;
      w[j] = *reinterpret_cast<const uint32_t *>(sm + row * 128 + ((((4 * ag) >> 4) ^ c) << 4) + ((4 * ag) & 15)) ^
             0x80808080u;
    }
    const bool full = T.na == TA && T.nb == TB;
    uint8_t *dp = T.dst + static_cast<int64_t>(4 * ag) * DaB + c * 16;
#pragma unroll
    for (int i = 0; i < 4; ++i, dp += DaB) {
      const int arow = 4 * ag + i;
      if (arow >= T.na)
        break;
      if constexpr (CH_ON == 1) {
        int64_t ch = T.a0 + arow;
        if (ch >= s.channel_length) {
          ok = false;
          ch = 0;
        }
        const float sc = s.param[ch], bi = 8388736.0f + static_cast<float>(zp_of(s, ch));
#pragma unroll
        for (int j = 0; j < VD; ++j) {
          ps[j] = sc;
          bias[j] = bi;
        }
      }
      float f[VD];
#pragma unroll
      for (int j = 0; j < VD; ++j)
        f[j] = __fmul_rn(__fsub_rn(__int_as_float(__byte_perm(w[j], 0x4B000000u, 0x7650 + i)), bias[j]), ps[j]);
      union {
        uint4 q;
        D e[VD];
        uint32_t u[4];
      } out;
      if constexpr (CHAIN == CH_DQ_F16) {
#pragma unroll
        for (int j = 0; j < VD; j += 2) {
          const __half2 h = __floats2half2_rn(f[j], f[j + 1]);
          out.u[j / 2] = *reinterpret_cast<const uint32_t *>(&h);
        }
      } else if constexpr (CHAIN == CH_DQ_BF16) {
#pragma unroll
        for (int j = 0; j < VD; j += 2) {
          const __nv_bfloat162 h = __floats2bfloat162_rn(f[j], f[j + 1]);
          out.u[j / 2] = *reinterpret_cast<const uint32_t *>(&h);
        }
      } else {
#pragma unroll
        for (int j = 0; j < VD; ++j)
          out.e[j] = static_cast<D>(__float_as_uint(f[j]));
      }
      if (full) {
        __stcs(reinterpret_cast<uint4 *>(dp), out.q);
      } else {
        for (int j = 0; j < VD; ++j)
          if (c * VD + j < T.nb)
            reinterpret_cast<D *>(dp)[j] = out.e[j];
      }
    }
    if (!ok)
      flag(d);
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// TMA-pipelined tile transposes, sm_100a: int8 -> f16/bf16 dequantize (the
// weight-fetch kernel) and 32-bit copies or f32 -> f16/bf16 casts.
//
// The source box is viewed by a 3-D tensor map (x = A cells, 128 bytes per
// box; y = group of 8 source rows, z = row within the group; strides 8*Sb and
// Sb), so one box of 128 bytes x 8 x 8 lands source row 8c+j at shared slot
// 8j+c. With the 128-byte swizzle (16-byte chunk index XOR slot mod 8) the
// store phase -- thread (ag, c) reads rows 8c..8c+7 at byte column 4*ag (four
// int8 cells or one 32-bit cell) -- hits 32 distinct banks.
//
// Warp roles: warps 0-7 convert and store, warp 8 produces. The producer keeps
// KStages tiles in flight in a ring of shared-memory stages, each with a
// `full` mbarrier (32 producer arrivals + the tile's byte count) and an
// `empty` mbarrier (one arrival per consumer warp). Per tile it waits for the
// stage to be empty, lane 0 arms `full` with the byte count and issues
// cp.async.bulk.tensor (plain tiled loads, no multicast; the source is this
// GPU's memory or, in the multi-GPU fetch, a peer's shard), then the lanes stage
// the tile's 64 per-column scales and biases next to it and arrive. Consumer
// warps wait on `full`, read the tile and its parameters into registers,
// release the stage and convert; there is no CTA-wide barrier in the loop, so
// warps drift up to KStages tiles apart instead of meeting every tile.
// Conversion and the 16-byte streaming stores are those of k_tile_s8.
//
// Every wait is bounded in time (TmaCtl::wait_ns of the global timer). A
// thread whose wait runs out sets the descriptor's fault word to 2 and leaves;
// thread 0 (or the producer) first waits, again bounded, for the copies that
// may still be in flight into this CTA's shared memory.
// ---------------------------------------------------------------------------

/// Per-launch controls of k_tma_tile: the time limit of each bounded wait and
/// the test hook's withheld job (UINT32_MAX: none; see sbc_test_withhold_tile).
struct TmaCtl {
  uint64_t wait_ns;
  uint32_t withhold_job;
};

// Ring depth and resident CTAs per SM of k_tma_tile (compile-time tuning
// points). Measured on the gate matrix (TB/s): 6 x 3 CTAs 5.00-5.03,
// 8 x 3 5.00-5.05, 4 x 4 4.92-4.96, 12 x 2 5.08-5.09, 10 x 2 5.08 (default:
// the same bytes in flight per SM as 12 x 2 with less shared memory).
#ifndef SBC_TMA_STAGES
#define SBC_TMA_STAGES 10
#endif
#ifndef SBC_TMA_CTAS_PER_SM
#define SBC_TMA_CTAS_PER_SM 2
#endif
constexpr int KStages = SBC_TMA_STAGES;
constexpr int KTmaTileBytes = 64 * 128;
constexpr int KTmaConsumers = 256;              // warps 0-7
constexpr int KTmaThreads = KTmaConsumers + 32; // + the producer warp

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}

/// Job order of k_tma_tile. Jobs walk groups of 2^lg source-column blocks (of
/// 128 bytes); inside a group the column block varies fastest, so the tiles
/// in flight at once read 2^lg * 128 contiguous bytes of each source row
/// while their outputs still cover whole runs of destination rows.
/// group.d = 2^lg * (source-row blocks of 64).
struct TileOrder {
  FastDiv group;
  uint32_t lg;
};

__device__ __forceinline__ void tile_of(uint32_t job, const TileOrder &o, uint32_t &ta, uint32_t &tb) {
  const uint32_t g = fdiv(job, o.group), r = job - g * o.group.d;
  ta = (g << o.lg) + (r & ((1u << o.lg) - 1));
  tb = r >> o.lg;
}

/// Shared-memory slot of parameter column n (0..63) of a tile: columns 32..63
/// swap their 16-byte halves, so the eight float4 reads of a warp (column
/// groups 8c..8c+3 or 8c+4..8c+7, c = 0..7) fall on 32 distinct banks.
__device__ __forceinline__ int param_slot(int n) { return n ^ (((n >> 5) & 1) << 2); }

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

/// Raise the phase's expected transaction bytes without arriving.
__device__ __forceinline__ void mbar_expect_tx_only(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}

/// 4-byte asynchronous global -> shared copy (tracked per thread).
__device__ __forceinline__ void cp_async4(void *dst_smem, const void *src_global) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_addr(dst_smem)),
               "l"(__cvta_generic_to_global(src_global))
               : "memory");
}

/// This thread's arrival on `bar`, made once all its earlier cp.async copies
/// completed (the barrier's expected count includes it: no increment).
__device__ __forceinline__ void cp_async_arrive(uint64_t *bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ bool mbar_try(uint32_t a, uint32_t parity) {
  uint32_t done;
  asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
               " selp.u32 %0, 1, 0, p;\n}"
               : "=r"(done)
               : "r"(a), "r"(parity)
               : "memory");
  return done != 0;
}

/// Wait for `parity` for at most `limit_ns` of the global timer (read only
/// once the first poll failed); true when the phase completed.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, uint64_t limit_ns) {
  const uint32_t a = smem_addr(bar);
  if (mbar_try(a, parity))
    return true;
  const uint64_t t0 = global_ns();
  for (;;) {
    if (mbar_try(a, parity))
      return true;
    if (global_ns() - t0 > limit_ns)
      return false;
  }
}

// Cache-policy tuning points of k_tma_tile: SBC_TMA_LOAD_EVICT_FIRST = 1
// marks the source boxes evict-first in L2 (they are read once);
// SBC_TMA_STORE = 0 streaming stores (st.global.cs), 1 L2-only (.cg),
// 2 write-back (default policy).
#ifndef SBC_TMA_LOAD_EVICT_FIRST
#define SBC_TMA_LOAD_EVICT_FIRST 0
#endif
#ifndef SBC_TMA_STORE
#define SBC_TMA_STORE 0
#endif

__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, int32_t x, int32_t y, int32_t z,
                                            uint64_t *bar) {
#if SBC_TMA_LOAD_EVICT_FIRST
  uint64_t policy;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
  asm volatile("cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
               " [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(smem_addr(dst)),
               "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_addr(bar)), "l"(policy)
               : "memory");
#else
  asm volatile("cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
               " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_addr(dst)),
               "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_addr(bar))
               : "memory");
#endif
}

/// A 16-byte result store of k_tma_tile (policy: SBC_TMA_STORE).
__device__ __forceinline__ void tma_out_store(uint4 *p, uint4 v) {
#if SBC_TMA_STORE == 1
  __stcg(p, v);
#elif SBC_TMA_STORE == 2
  *p = v;
#else
  __stcs(p, v);
#endif
}

/// Tensor maps of the sources of one k_tma_tile launch: source j (a block of
/// consecutive source rows, possibly in another GPU's memory) holds the
/// b-tiles [tb_first[j], tb_first[j + 1]). One source in the common case;
/// several when a multi-GPU fetch's shards are read in place.
constexpr int kMaxTmaSources = 8;
struct TmaSources {
  CUtensorMap map[kMaxTmaSources];
  uint32_t tb_first[kMaxTmaSources + 1];
  int32_t n;
};

/// WS = 1: int8 source, CHAIN CH_DQ_F16 / CH_DQ_BF16 (f16/bf16 result), tiles
/// of 128 A x 64 B cells. WS = 4: 32-bit source, CHAIN CH_COPY (32-bit
/// result) or CH_F16 / CH_BF16, CH_ON = 0, tiles of 32 A x 64 B cells. Both
/// move one 8 KB box per tile through the same shared-memory layout.
template <int WS, int CHAIN, int CH_ON>
__global__ void __launch_bounds__(KTmaThreads, SBC_TMA_CTAS_PER_SM) k_tma_tile(const __grid_constant__ TmaSources srcs,
                                                             const __grid_constant__ sbc_relocate d, TileOrder ord,
                                                             uint32_t tiles, TmaCtl ctl) {
  constexpr int TB = 64, VD = 8;
  constexpr int TA = 128 / WS;                     // A cells per tile
  constexpr int WD = CHAIN == CH_COPY ? WS : 2;    // result bytes per cell
  // Rows per group of the tensor-map view (source row GR*y + z lands at slot
  // z * (64 / GR) + y). 32-bit copies use groups of 4: thread c then reads
  // rows 4c..4c+3 and 32+4c..32+4c+3 (slots 16j + c and 16j + 8 + c, still 8
  // distinct swizzle phases) and its two 16-byte stores each join the other
  // threads of its row in one contiguous 128-byte segment.
  constexpr int GR = (WS == 4 && CHAIN == CH_COPY) ? 4 : 8;
  static_assert(WS == 1 || CH_ON == 0, "32-bit tiles carry no parameters");
  extern __shared__ __align__(1024) uint8_t dyn[];
  __shared__ __align__(8) uint64_t full[KStages], empty[KStages];
  // Per-column dequantize parameters of the tile in each stage (CH_ON == 2):
  // scales, and zero points when they are per channel.
  __shared__ __align__(16) float s_scale[KStages][64];
  __shared__ __align__(16) int32_t s_zp[KStages][64];
  __shared__ int timed_out;
  uint8_t *stage0 = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(dyn) + 1023) & ~uintptr_t(1023));
  const int t = threadIdx.x;
  const sbc_stage &s = d.stages[0];
  const uint32_t G = gridDim.x;

  if (t == 0) {
    for (int i = 0; i < KStages; ++i) {
      mbar_init(&full[i], 32);
      mbar_init(&empty[i], KTmaConsumers / 32);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    timed_out = 0;
  }
  __syncthreads(); // the only CTA-wide barrier
  // The fault word may be mapped host memory: a plain store made visible
  // system-wide (only the value 2 is ever written, so no atomic is needed).
  auto fail = [&]() {
    if (atomicExch(&timed_out, 1) == 0 && d.fault) {
      *reinterpret_cast<volatile int32_t *>(d.fault) = 2;
      __threadfence_system();
    }
  };
  // Bounded wait for the copies of local tiles [lo, hi) (issued, maybe in flight).
  auto drain = [&](uint32_t lo, uint32_t hi) {
    for (uint32_t q = lo; q < hi && blockIdx.x + q * G < tiles; ++q)
      mbar_wait(&full[q % KStages], (q / KStages) & 1, ctl.wait_ns);
  };

  if (t >= KTmaConsumers) { // ---- producer warp
    const int lane = t - KTmaConsumers;
    if (lane < srcs.n)
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&srcs.map[lane])) : "memory");
    uint32_t k = 0;
    for (;; ++k) {
      const uint32_t job = blockIdx.x + k * G;
      if (job >= tiles)
        break;
      const int st = k % KStages;
      if (k >= KStages && !mbar_wait(&empty[st], (k / KStages - 1) & 1, ctl.wait_ns)) {
        fail();
        drain(k - KStages, k); // every lane: its own parameter copies land before it leaves
        return;
      }
      if (job == ctl.withhold_job) {
        // test hook: neither the copy nor any arrival, so this tile's
        // consumers run out of their bounded wait
        continue;
      }
      uint32_t ta, tb;
      tile_of(job, ord, ta, tb);
      if constexpr (CH_ON == 2) {
        // This lane's two parameter columns go straight from global to the
        // stage's shared slots by cp.async, and its arrival on `full` is
        // made when they have landed: the producer never waits for a global
        // load. Columns past the table read entry 0 (the consumers flag the
        // tile).
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          int64_t ch = d.box_lo[1] + static_cast<int64_t>(tb) * TB + lane + 32 * h;
          if (ch >= s.channel_length)
            ch = 0;
          cp_async4(&s_scale[st][param_slot(lane + 32 * h)], s.param + ch);
          if (s.zp_mode == 2)
            cp_async4(&s_zp[st][param_slot(lane + 32 * h)], s.zero_point + ch);
        }
      }
      if (lane == 0) {
        int j = 0; // the source holding b-tile tb
        while (j + 1 < srcs.n && tb >= srcs.tb_first[j + 1])
          ++j;
        if constexpr (CH_ON == 2)
          mbar_expect_tx_only(&full[st], KTmaTileBytes); // lane 0 arrives below, with the other lanes
        else
          mbar_expect_tx(&full[st], KTmaTileBytes); // lane 0's arrival
        tma_load_3d(stage0 + st * KTmaTileBytes, &srcs.map[j], static_cast<int32_t>(ta * TA),
                    static_cast<int32_t>((tb - srcs.tb_first[j]) * (TB / GR)), 0, &full[st]);
      }
      if constexpr (CH_ON == 2)
        cp_async_arrive(&full[st]); // once this lane's parameter copies landed
      else if (lane != 0)
        mbar_arrive(&full[st]);
    }
    // A lane leaves only after its parameter copies of the last tiles landed
    // (the stage's phase completes after every lane's copies).
    if constexpr (CH_ON == 2)
      drain(k > KStages ? k - KStages : 0, k);
    return;
  }

  // ---- consumer warps
  const int ag = t >> 3, c = t & 7;
  const int64_t Da = d.dst_strides[0], DaB = Da * WD;
  uint8_t *const dst0 = static_cast<uint8_t *>(d.dst) - d.dst_offset * WD;
  float ps[VD], bias[VD];
  // 2^23 + 128 + zero point: the int8 -> f32 conversion's bias; the same for
  // every column unless the zero points are per channel.
  float bias_all = 0.0f;
  if constexpr (WS == 1)
    bias_all = 8388736.0f + static_cast<float>(s.zp_mode == 1 ? s.zero_point[0] : 0);
  if constexpr (WS == 1 && CH_ON == 0) {
#pragma unroll
    for (int j = 0; j < VD; ++j) {
      ps[j] = s.param[0];
      bias[j] = bias_all;
    }
  }
  for (uint32_t k = 0;; ++k) {
    const uint32_t job = blockIdx.x + k * G;
    if (job >= tiles)
      break;
    const int st = k % KStages;
    if (!mbar_wait(&full[st], (k / KStages) & 1, ctl.wait_ns)) {
      fail();
      if (t == 0) // the producer cannot pass tile k + KStages - 1 before this warp releases tile k
        drain(k, k + KStages);
      return;
    }
    uint32_t ta, tb;
    tile_of(job, ord, ta, tb);
    bool ok = true;
    if constexpr (CH_ON == 2) {
      const int lo = param_slot(c * VD), hi = param_slot(c * VD + 4);
      const float4 s0 = *reinterpret_cast<const float4 *>(&s_scale[st][lo]);
      const float4 s1 = *reinterpret_cast<const float4 *>(&s_scale[st][hi]);
      ps[0] = s0.x, ps[1] = s0.y, ps[2] = s0.z, ps[3] = s0.w, ps[4] = s1.x, ps[5] = s1.y, ps[6] = s1.z, ps[7] = s1.w;
      if (s.zp_mode == 2) {
        const int4 z0 = *reinterpret_cast<const int4 *>(&s_zp[st][lo]);
        const int4 z1 = *reinterpret_cast<const int4 *>(&s_zp[st][hi]);
        const int z[VD] = {z0.x, z0.y, z0.z, z0.w, z1.x, z1.y, z1.z, z1.w};
#pragma unroll
        for (int j = 0; j < VD; ++j)
          bias[j] = 8388736.0f + static_cast<float>(z[j]);
      } else {
#pragma unroll
        for (int j = 0; j < VD; ++j)
          bias[j] = bias_all;
      }
      // a column past the parameter table (its copy read entry 0) flags the tile
      ok = d.box_lo[1] + static_cast<int64_t>(tb) * TB + (TB - 1) < s.channel_length;
    }
    const int64_t a0 = d.box_lo[0] + static_cast<int64_t>(ta) * TA;
    const int64_t b0 = d.box_lo[1] + static_cast<int64_t>(tb) * TB;
    const uint8_t *sp = stage0 + st * KTmaTileBytes;
    uint32_t w[VD];
#pragma unroll
    for (int j = 0; j < VD; ++j) {
      // GR == 8: word j = source row 8c + j; GR == 4: rows 4c + j (j < 4), 32 + 4c + (j - 4)
      const int slot = GR == 8 ? j * 8 + c : (j & 3) * 16 + (j >> 2) * 8 + c;
      w[j] = *reinterpret_cast<const uint32_t *>(sp + slot * 128 + ((((4 * ag) >> 4) ^ c) << 4) + ((4 * ag) & 15));
    }
    __syncwarp();
    if ((t & 31) == 0)
      mbar_arrive(&empty[st]); // this warp is done with the stage
    if constexpr (WS == 4 && GR == 4) {
      // words 0-3: cells (a0 + ag, b0 + 4c + j); words 4-7: cells b0 + 32 + 4c + j
      uint4 *dp = reinterpret_cast<uint4 *>(dst0 + (a0 * Da + b0) * WD + static_cast<int64_t>(ag) * DaB + c * 16);
      __stcs(dp, make_uint4(w[0], w[1], w[2], w[3]));
      __stcs(dp + 8, make_uint4(w[4], w[5], w[6], w[7]));
      continue;
    } else if constexpr (WS == 4) {
      // cell (a0 + ag, b0 + 8c + j) is word j: one result row segment of 8 cells
      uint4 out[WD / 2];
      uint32_t *u = reinterpret_cast<uint32_t *>(out);
#pragma unroll
      for (int j = 0; j < VD; ++j) {
        if constexpr (CHAIN == CH_COPY)
          u[j] = w[j];
        else if constexpr (CHAIN == CH_F16)
          reinterpret_cast<uint16_t *>(u)[j] = static_cast<uint16_t>(narrow_f16(w[j]));
        else
          reinterpret_cast<uint16_t *>(u)[j] = static_cast<uint16_t>(narrow_bf16(w[j]));
      }
      uint4 *dp = reinterpret_cast<uint4 *>(dst0 + (a0 * Da + b0) * WD + static_cast<int64_t>(ag) * DaB +
                                            c * VD * WD);
#pragma unroll
      for (int h = 0; h < WD / 2; ++h)
        __stcs(dp + h, out[h]);
      continue;
    } else {
#pragma unroll
      for (int j = 0; j < VD; ++j)
        w[j] ^= 0x80808080u;
    }
    uint8_t *dp = dst0 + (a0 * Da + b0) * 2 + static_cast<int64_t>(4 * ag) * DaB + c * 16;
#pragma unroll
    for (int i = 0; i < 4; ++i, dp += DaB) {
      if constexpr (CH_ON == 1) {
        int64_t ch = a0 + 4 * ag + i;
        if (ch >= s.channel_length) {
          ok = false;
          ch = 0;
        }
        const float sc = s.param[ch], bi = 8388736.0f + static_cast<float>(zp_of(s, ch));
#pragma unroll
        for (int j = 0; j < VD; ++j) {
          ps[j] = sc;
          bias[j] = bi;
        }
      }
      // Two columns at a time on the packed f32x2 pipe: (x - bias) then
      // * scale, each an IEEE round-to-nearest-even operation per lane (the
      // same results as the scalar __fsub_rn / __fmul_rn, half the
      // instructions).
      uint4 out;
      uint32_t *u = reinterpret_cast<uint32_t *>(&out);
#pragma unroll
      for (int j = 0; j < VD; j += 2) {
        const float2 x = make_float2(__int_as_float(__byte_perm(w[j], 0x4B000000u, 0x7650 + i)),
                                     __int_as_float(__byte_perm(w[j + 1], 0x4B000000u, 0x7650 + i)));
        const float2 f = __fmul2_rn(__fadd2_rn(x, make_float2(-bias[j], -bias[j + 1])),
                                    make_float2(ps[j], ps[j + 1]));
        if constexpr (CHAIN == CH_DQ_BF16) {
          const __nv_bfloat162 h = __floats2bfloat162_rn(f.x, f.y);
          u[j / 2] = *reinterpret_cast<const uint32_t *>(&h);
        } else {
          const __half2 h = __floats2half2_rn(f.x, f.y);
          u[j / 2] = *reinterpret_cast<const uint32_t *>(&h);
        }
      }
      tma_out_store(reinterpret_cast<uint4 *>(dp), out);
    }
    if (!ok)
      flag(d);
  }
}

// ---------------------------------------------------------------------------
// Tall int8 tiles: 128 A cells x 128 source rows per tile (16 KB boxes), so
// every destination row segment a tile writes is 128 f16 = 256 bytes. The
// 32-bit tile kernel, which writes 256-byte segments, reaches ~0.96 of the
// copy peak where the 64-row int8 tile (128-byte segments) stays at ~0.77.
//
// The box is the same 3-D view with y = 16 groups of 8 rows: source row
// 8y + z lands at shared slot 16z + y (128 bytes each, 128-byte swizzle).
// Consumer thread (ag, c), ag and c in 0..15, owns destination rows
// a0 + 8ag + i (i < 8) and columns b0 + 8c + j (j < 8): it reads the 8 bytes
// at column 8ag of source rows 8c + j (slots 16j + c). Lanes are laid out so
// that each half-warp covers c mod 8 and ag mod 2 once: its sixteen 8-byte
// reads hit 32 distinct banks; each store instruction of a warp writes two
// destination rows x 256 contiguous bytes. Producer, barriers, bounded waits,
// fault word and the test hook are those of k_tma_tile. With DYN the tiles
// are taken in the dynamic order below (the producer passes each stage's
// tile index to the consumers through shared memory, and an end marker
// after the last one) instead of the persistent grid's round robin.
// ---------------------------------------------------------------------------

// Ring depth of k_tma_tall (16 KB stages, 2 CTAs per SM). Gate matrix
// [28672, 8192] per launch: 4 stages 0.1275 ms, 5 stages 0.1285 ms, 6 stages
// 0.1292 ms; the 64-row k_tma_tile on the same box 0.1417-0.1434 ms.
#ifndef SBC_TMA_TALL_STAGES
#define SBC_TMA_TALL_STAGES 4
#endif
constexpr int KTallStages = SBC_TMA_TALL_STAGES;
constexpr int KTallTileBytes = 128 * 128;

// Dynamic tile order (cluster launch control). The grid has one CTA per
// tile; a running CTA asks the hardware to cancel the launch of a CTA that
// has not started yet (clusterlaunchcontrol.try_cancel, one CTA per cluster,
// no multicast) and takes over its tile, until a request fails. Every tile is
// then done exactly once -- by its own CTA if that CTA launched, else by the
// CTA that cancelled it -- and SMs that run faster take more tiles, instead
// of each CTA owning a fixed 1/G of them.

/// Arm `bar` for a 16-byte response and request the cancellation of one
/// CTA not yet launched; the response lands in `resp`.
__device__ __forceinline__ void clc_request(uint4 *resp, uint64_t *bar) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], 16;" ::"r"(smem_addr(bar)) : "memory");
  asm volatile("clusterlaunchcontrol.try_cancel.async.shared::cta.mbarrier::complete_tx::bytes.b128 [%0], [%1];" ::"r"(
                   smem_addr(resp)),
               "r"(smem_addr(bar))
               : "memory");
}

/// The x index of the CTA a completed request cancelled, or UINT32_MAX if
/// the request failed (no CTA left to cancel: no request may follow).
__device__ __forceinline__ uint32_t clc_result(const uint4 *resp) {
  uint32_t x = UINT32_MAX, ok = 0;
  asm volatile("{\n .reg .pred p;\n .reg .b128 r;\n ld.shared.b128 r, [%2];\n"
               " clusterlaunchcontrol.query_cancel.is_canceled.pred.b128 p, r;\n"
               " selp.u32 %1, 1, 0, p;\n"
               " @p clusterlaunchcontrol.query_cancel.get_first_ctaid::x.b32.b128 %0, r;\n}"
               : "+r"(x), "=r"(ok)
               : "r"(smem_addr(resp))
               : "memory");
  // the next response into this buffer is an async-proxy write after this read
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  return ok ? x : UINT32_MAX;
}

constexpr uint32_t kNoTile = UINT32_MAX; // end marker of the dynamic order

template <int CHAIN, int CH_ON, bool DYN>
__global__ void __launch_bounds__(KTmaThreads, SBC_TMA_CTAS_PER_SM) k_tma_tall(const __grid_constant__ TmaSources srcs,
                                                             const __grid_constant__ sbc_relocate d, TileOrder ord,
                                                             uint32_t tiles, TmaCtl ctl) {
  constexpr int TA = 128, TB = 128, VD = 8, GR = 8;
  // Arrivals that complete a stage: the 32 producer lanes; with the dynamic
  // order and cp.async parameters, lane 0 also arrives once (a release, after
  // it wrote the stage's tile index) besides its cp.async arrival.
  constexpr uint32_t FullCount = (DYN && CH_ON == 2) ? 33 : 32;
  extern __shared__ __align__(1024) uint8_t dyn[];
  __shared__ __align__(8) uint64_t full[KTallStages], empty[KTallStages];
  __shared__ __align__(16) float s_scale[KTallStages][TB];
  __shared__ __align__(16) int32_t s_zp[KTallStages][TB];
  __shared__ uint32_t s_job[KTallStages]; // DYN: the tile of each stage (kNoTile: the end)
  __shared__ __align__(16) uint4 clc_resp[2];
  __shared__ __align__(8) uint64_t clc_bar[2];
  __shared__ int timed_out;
  uint8_t *stage0 = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(dyn) + 1023) & ~uintptr_t(1023));
  const int t = threadIdx.x;
  const sbc_stage &s = d.stages[0];
  const uint32_t G = gridDim.x;

  if (t == 0) {
    for (int i = 0; i < KTallStages; ++i) {
      mbar_init(&full[i], FullCount);
      mbar_init(&empty[i], KTmaConsumers / 32);
    }
    mbar_init(&clc_bar[0], 1);
    mbar_init(&clc_bar[1], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    timed_out = 0;
  }
  __syncthreads(); // the only CTA-wide barrier
  auto fail = [&]() {
    if (atomicExch(&timed_out, 1) == 0 && d.fault) {
      *reinterpret_cast<volatile int32_t *>(d.fault) = 2;
      __threadfence_system();
    }
  };
  // Bounded wait for the copies of local tiles [lo, hi) (issued, maybe in flight).
  auto drain = [&](uint32_t lo, uint32_t hi) {
    for (uint32_t q = lo; q < hi && (DYN || blockIdx.x + q * G < tiles); ++q)
      mbar_wait(&full[q % KTallStages], (q / KTallStages) & 1, ctl.wait_ns);
  };

  if (t >= KTmaConsumers) { // ---- producer warp
    const int lane = t - KTmaConsumers;
    if (lane < srcs.n)
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&srcs.map[lane])) : "memory");
    uint32_t job = blockIdx.x;
    uint32_t asked = 0; // DYN: cancellation requests issued (request r uses buffer r & 1)
    if constexpr (DYN) {
      if (lane == 0)
        clc_request(&clc_resp[0], &clc_bar[0]);
      asked = 1;
    }
    // DYN: bounded wait for an outstanding cancellation response before leaving
    auto settle = [&]() {
      if constexpr (DYN) {
        if (asked > 0 && job != kNoTile)
          mbar_wait(&clc_bar[(asked - 1) & 1], ((asked - 1) >> 1) & 1, ctl.wait_ns);
      }
    };
    uint32_t k = 0;
    for (;; ++k) {
      if constexpr (!DYN) {
        job = blockIdx.x + k * G;
        if (job >= tiles)
          break;
      }
      const int st = k % KTallStages;
      if (k >= KTallStages && !mbar_wait(&empty[st], (k / KTallStages - 1) & 1, ctl.wait_ns)) {
        fail();
        drain(k - KTallStages, k);
        settle();
        return;
      }
      if constexpr (DYN) {
        if (job == kNoTile) { // the end: consumers leave at this stage
          if (lane == 0) {
            s_job[st] = kNoTile;
            asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(&full[st])),
                         "r"(FullCount)
                         : "memory");
          }
          break;
        }
      }
      if (job != ctl.withhold_job) { // test hook: no copy and no arrival for the withheld tile
        uint32_t ta, tb;
        tile_of(job, ord, ta, tb);
        if constexpr (CH_ON == 2) {
#pragma unroll
          for (int h = 0; h < TB / 32; ++h) {
            int64_t ch = d.box_lo[1] + static_cast<int64_t>(tb) * TB + lane + 32 * h;
            if (ch >= s.channel_length)
              ch = 0;
            cp_async4(&s_scale[st][param_slot(lane + 32 * h)], s.param + ch);
            if (s.zp_mode == 2)
              cp_async4(&s_zp[st][param_slot(lane + 32 * h)], s.zero_point + ch);
          }
        }
        if (lane == 0) {
          int j = 0;
          while (j + 1 < srcs.n && tb >= srcs.tb_first[j + 1])
            ++j;
          if constexpr (DYN)
            s_job[st] = job; // published by lane 0's arrival below (release)
          if constexpr (CH_ON == 2 && !DYN)
            mbar_expect_tx_only(&full[st], KTallTileBytes);
          else
            mbar_expect_tx(&full[st], KTallTileBytes);
          tma_load_3d(stage0 + st * KTallTileBytes, &srcs.map[j], static_cast<int32_t>(ta * TA),
                      static_cast<int32_t>((tb - srcs.tb_first[j]) * (TB / GR)), 0, &full[st]);
        }
        if constexpr (CH_ON == 2)
          cp_async_arrive(&full[st]);
        else if (lane != 0)
          mbar_arrive(&full[st]);
      }
      if constexpr (DYN) { // the next tile: the outstanding request's answer
        const uint32_t r = asked - 1;
        if (!mbar_wait(&clc_bar[r & 1], (r >> 1) & 1, ctl.wait_ns)) {
          fail();
          drain(k + 1 > KTallStages ? k + 1 - KTallStages : 0, k + 1);
          return;
        }
        job = clc_result(&clc_resp[r & 1]);
        __syncwarp(); // every lane read the response before its buffer is reused
        if (job != kNoTile) {
          if (lane == 0)
            clc_request(&clc_resp[asked & 1], &clc_bar[asked & 1]);
          ++asked;
        }
      }
    }
    // A lane leaves once its own parameter copies have landed. (Not by waiting
    // on the last stages' barriers: with the dynamic order the end marker's
    // stage reuses the barrier of the oldest of them, whose awaited phase
    // would then already be two phases back.)
    if constexpr (CH_ON == 2)
      asm volatile("cp.async.wait_all;" ::: "memory");
    return;
  }

  // ---- consumer warps
  const int lane = t & 31;
  const int c = (lane & 7) | (((lane >> 4) & 1) << 3);  // 0..15
  const int ag = 2 * (t >> 5) + ((lane >> 3) & 1);      // 0..15
  const int64_t Da = d.dst_strides[0], DaB = Da * 2;
  uint8_t *const dst0 = static_cast<uint8_t *>(d.dst) - d.dst_offset * 2;
  const float bias_all = 8388736.0f + static_cast<float>(s.zp_mode == 1 ? s.zero_point[0] : 0);
  float ps[VD], bias[VD];
  if constexpr (CH_ON == 0) {
#pragma unroll
    for (int j = 0; j < VD; ++j) {
      ps[j] = s.param[0];
      bias[j] = bias_all;
    }
  }
  for (uint32_t k = 0;; ++k) {
    uint32_t job = blockIdx.x + k * G;
    if (!DYN && job >= tiles)
      break;
    const int st = k % KTallStages;
    if (!mbar_wait(&full[st], (k / KTallStages) & 1, ctl.wait_ns)) {
      fail();
      if (t == 0)
        drain(k, k + KTallStages);
      return;
    }
    if constexpr (DYN) {
      job = *reinterpret_cast<volatile uint32_t *>(&s_job[st]);
      if (job == kNoTile)
        break;
    }
    uint32_t ta, tb;
    tile_of(job, ord, ta, tb);
    bool ok = true;
    if constexpr (CH_ON == 2) {
      const int lo = param_slot(c * VD), hi = param_slot(c * VD + 4);
      const float4 s0 = *reinterpret_cast<const float4 *>(&s_scale[st][lo]);
      const float4 s1 = *reinterpret_cast<const float4 *>(&s_scale[st][hi]);
      ps[0] = s0.x, ps[1] = s0.y, ps[2] = s0.z, ps[3] = s0.w, ps[4] = s1.x, ps[5] = s1.y, ps[6] = s1.z, ps[7] = s1.w;
      if (s.zp_mode == 2) {
        const int4 z0 = *reinterpret_cast<const int4 *>(&s_zp[st][lo]);
        const int4 z1 = *reinterpret_cast<const int4 *>(&s_zp[st][hi]);
        const int z[VD] = {z0.x, z0.y, z0.z, z0.w, z1.x, z1.y, z1.z, z1.w};
#pragma unroll
        for (int j = 0; j < VD; ++j)
          bias[j] = 8388736.0f + static_cast<float>(z[j]);
      } else {
#pragma unroll
        for (int j = 0; j < VD; ++j)
          bias[j] = bias_all;
      }
      ok = d.box_lo[1] + static_cast<int64_t>(tb) * TB + (TB - 1) < s.channel_length;
    }
    const int64_t a0 = d.box_lo[0] + static_cast<int64_t>(ta) * TA;
    const int64_t b0 = d.box_lo[1] + static_cast<int64_t>(tb) * TB;
    const uint8_t *sp = stage0 + st * KTallTileBytes;
    // bytes 8ag..8ag+7 of source rows 8c + j (slot 16j + c; slot mod 8 = c mod 8)
    uint2 w[VD];
    const int chunk = ((ag >> 1) ^ (c & 7)) << 4, half = (ag & 1) << 3;
#pragma unroll
    for (int j = 0; j < VD; ++j)
      w[j] = *reinterpret_cast<const uint2 *>(sp + (16 * j + c) * 128 + chunk + half);
    __syncwarp();
    if (lane == 0)
      mbar_arrive(&empty[st]); // this warp is done with the stage
#pragma unroll
    for (int j = 0; j < VD; ++j) {
      w[j].x ^= 0x80808080u;
      w[j].y ^= 0x80808080u;
    }
    uint8_t *dp = dst0 + (a0 * Da + b0) * 2 + static_cast<int64_t>(8 * ag) * DaB + c * 16;
#pragma unroll
    for (int i = 0; i < VD; ++i, dp += DaB) {
      if constexpr (CH_ON == 1) {
        int64_t ch = a0 + 8 * ag + i;
        if (ch >= s.channel_length) {
          ok = false;
          ch = 0;
        }
        const float sc = s.param[ch], bi = 8388736.0f + static_cast<float>(zp_of(s, ch));
#pragma unroll
        for (int j = 0; j < VD; ++j) {
          ps[j] = sc;
          bias[j] = bi;
        }
      }
      uint4 out;
      uint32_t *u = reinterpret_cast<uint32_t *>(&out);
#pragma unroll
      for (int j = 0; j < VD; j += 2) {
        const uint32_t wa = i < 4 ? w[j].x : w[j].y, wb = i < 4 ? w[j + 1].x : w[j + 1].y;
        const float2 x = make_float2(__int_as_float(__byte_perm(wa, 0x4B000000u, 0x7650 + (i & 3))),
                                     __int_as_float(__byte_perm(wb, 0x4B000000u, 0x7650 + (i & 3))));
        const float2 f = __fmul2_rn(__fadd2_rn(x, make_float2(-bias[j], -bias[j + 1])),
                                    make_float2(ps[j], ps[j + 1]));
        if constexpr (CHAIN == CH_DQ_BF16) {
          const __nv_bfloat162 h = __floats2bfloat162_rn(f.x, f.y);
          u[j / 2] = *reinterpret_cast<const uint32_t *>(&h);
        } else {
          const __half2 h = __floats2half2_rn(f.x, f.y);
          u[j / 2] = *reinterpret_cast<const uint32_t *>(&h);
        }
      }
      tma_out_store(reinterpret_cast<uint4 *>(dp), out);
    }
    if (!ok)
      flag(d);
  }
}

// ---------------------------------------------------------------------------
// Fill
// ---------------------------------------------------------------------------


template <int W>
__global__ void __launch_bounds__(256) k_fill(void *dst, int64_t count, uint64_t bits) {
  using D = typename Word<W>::T;
  D *p = static_cast<D *>(dst);
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < count;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    p[i] = static_cast<D>(bits);
}

// ---------------------------------------------------------------------------
// Host side: chain detection, dispatch over the instantiations, launch shape.
// ---------------------------------------------------------------------------

int chain_of(const sbc_relocate &d) {
  if (d.nstages == 0)
    return CH_COPY;
  const int o0 = d.stages[0].op;
  if (d.nstages == 1) {
    switch (o0) {
    case SBC_QUANTIZE: return CH_Q;
    case SBC_DEQUANTIZE: return CH_DQ;
    case SBC_NARROW_F16: return CH_F16;
    case SBC_NARROW_BF16: return CH_BF16;
    case SBC_WIDEN_F16: return CH_W16;
    case SBC_WIDEN_BF16: return CH_WB16;
    }
  }
  if (d.nstages == 2 && o0 == SBC_DEQUANTIZE && d.stages[1].channel == SBC_CH_NONE) {
    if (d.stages[1].op == SBC_NARROW_F16)
      return CH_DQ_F16;
    if (d.stages[1].op == SBC_NARROW_BF16)
      return CH_DQ_BF16;
  }
  return CH_ANY;
}

/// Channel kinds a specialized chain may use (it only reads stage 0).
bool chain_channels_ok(const sbc_relocate &d, int chain, bool allow_offset) {
  for (int k = 0; k < d.nstages; ++k) {
    const int ch = d.stages[k].channel;
    if (ch == SBC_CH_EXPR || (ch == SBC_CH_OFFSET && !allow_offset))
      return false;
  }
  (void)chain;
  return true;
}

int g_sms = 0;
int sm_count() {
  if (g_sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_sms, cudaDevAttrMultiProcessorCount, dev);
    if (g_sms <= 0)
      g_sms = 148;
  }
  return g_sms;
}

int64_t grid_for(int64_t work_items, int per_block, int blocks_per_sm) {
  int64_t blocks = (work_items + per_block - 1) / per_block;
  const int64_t cap = static_cast<int64_t>(sm_count()) * blocks_per_sm;
  if (blocks > cap)
    blocks = cap;
  return blocks < 1 ? 1 : blocks;
}

int launched(cudaError_t e) {
  if (e == cudaSuccess)
    e = cudaGetLastError();
  if (e == cudaSuccess)
    g_launches.fetch_add(1, std::memory_order_relaxed);
  return static_cast<int>(e);
}

template <template <int, int, int> class F, typename... Args>
int dispatch(int ws, int wd, int chain, Args &&...args) {
#define SBC_CASE(WS_, WD_, CH_)                                                                                 \
  if (ws == WS_ && wd == WD_ && chain == CH_)                                                                  \
    return F<WS_, WD_, CH_>::run(args...);
  SBC_CASE(1, 1, CH_COPY)
  SBC_CASE(2, 2, CH_COPY)
  SBC_CASE(4, 4, CH_COPY)
  SBC_CASE(8, 8, CH_COPY)
  SBC_CASE(4, 1, CH_Q)
  SBC_CASE(1, 4, CH_DQ)
  SBC_CASE(4, 2, CH_F16)
  SBC_CASE(4, 2, CH_BF16)
  SBC_CASE(2, 4, CH_W16)
  SBC_CASE(2, 4, CH_WB16)
  SBC_CASE(1, 2, CH_DQ_F16)
  SBC_CASE(1, 2, CH_DQ_BF16)
  SBC_CASE(1, 1, CH_ANY)
  SBC_CASE(1, 2, CH_ANY)
  SBC_CASE(1, 4, CH_ANY)
  SBC_CASE(2, 1, CH_ANY)
  SBC_CASE(2, 2, CH_ANY)
  SBC_CASE(2, 4, CH_ANY)
  SBC_CASE(4, 1, CH_ANY)
  SBC_CASE(4, 2, CH_ANY)
  SBC_CASE(4, 4, CH_ANY)
#undef SBC_CASE
  return SBC_EUNSUPPORTED;
}

template <int WS, int WD, int CH> struct GenericLaunch {
  static int run(const sbc_relocate &d, int64_t total, cudaStream_t s) {
    const int64_t blocks = grid_for(total, 256, 8);
    k_generic<WS, WD, CH><<<static_cast<unsigned>(blocks), 256, 0, s>>>(d, total);
    return launched(cudaSuccess);
  }
};

template <int WS, int WD, int CH> struct ContiguousLaunch {
  static int run(const sbc_relocate &d, int64_t vbegin, int64_t nunits, ScalarEnds ends, cudaStream_t s) {
    if constexpr (WS == 8 || WD == 8) {
      return SBC_EUNSUPPORTED;
    } else {
      constexpr int R = Units<WS, WD>::R;
      const int64_t blocks = grid_for((nunits + R - 1) / R, 256, 8); // a thread takes R units
      // the ends' code is compiled in only where there are ends (it cost the
      // aligned body 5 % when always present)
      if (ends.nhead + ends.ntail)
        k_contiguous<WS, WD, CH, true><<<static_cast<unsigned>(blocks), 256, 0, s>>>(d, vbegin, nunits, ends);
      else
        k_contiguous<WS, WD, CH, false><<<static_cast<unsigned>(blocks), 256, 0, s>>>(d, vbegin, nunits, ends);
      return launched(cudaSuccess);
    }
  }
};

template <int WS, int WD, int CH> struct TransposeLaunch {
  static int run(const sbc_relocate &d, int ta, int tb, int64_t tiles_a, int64_t tiles_b, int64_t nbatch,
                 cudaStream_t s) {
    if constexpr (WS == 8) {
      return SBC_EUNSUPPORTED;
    } else {
      const size_t smem = static_cast<size_t>(ta) * (tb + 1) * WD;
      const int64_t jobs = tiles_a * tiles_b * nbatch;
      int64_t blocks = jobs;
      const int64_t cap = static_cast<int64_t>(sm_count()) * 16;
      if (blocks > cap)
        blocks = cap;
      k_transpose<WS, WD, CH><<<static_cast<unsigned>(blocks), 256, smem, s>>>(d, ta, tb, tiles_a, tiles_b, nbatch);
      return launched(cudaSuccess);
    }
  }
};

FastDiv make_fastdiv(uint32_t dv) {
  FastDiv f;
  uint32_t l = 0;
  while ((1ull << l) < dv)
    ++l;
  f.s = 31 + l;
  f.d = dv;
  f.m = ((1ull << f.s) + dv - 1) / dv;
  return f;
}

/// TMA path switch: on unless SYM_B200_TMA=0 (kept for A/B measurement).
bool tma_enabled() {
  static const bool on = [] {
    const char *v = std::getenv("SYM_B200_TMA");
    return !(v && v[0] == '0');
  }();
  return on;
}

#ifndef SBC_TMA_TALL_DEFAULT
#define SBC_TMA_TALL_DEFAULT 1
#endif
/// Whether int8 tiles of 128 source rows (k_tma_tall) are used where the
/// shapes allow (SYM_B200_TMA_TALL=0/1; default SBC_TMA_TALL_DEFAULT).
bool tma_tall_enabled() {
  static const bool on = [] {
    const char *v = std::getenv("SYM_B200_TMA_TALL");
    return v ? v[0] != '0' : SBC_TMA_TALL_DEFAULT != 0;
  }();
  return on;
}

// Measured on the gate matrix [28672, 8192] per launch (two runs each):
// fixed round robin 0.1281 / 0.1283 ms, dynamic order 0.1173 / 0.1171 ms.
#ifndef SBC_TMA_DYNAMIC_DEFAULT
#define SBC_TMA_DYNAMIC_DEFAULT 1
#endif
/// Whether k_tma_tall takes its tiles in the dynamic order (one CTA per tile,
/// cluster launch control) instead of a persistent grid's fixed round robin
/// (SYM_B200_TMA_DYNAMIC=0/1; default SBC_TMA_DYNAMIC_DEFAULT).
bool tma_dynamic_enabled() {
  static const bool on = [] {
    const char *v = std::getenv("SYM_B200_TMA_DYNAMIC");
    return v ? v[0] != '0' : SBC_TMA_DYNAMIC_DEFAULT != 0;
  }();
  return on;
}

/// Controls of one launch of a kernel with bounded waits: the current time
/// limit, and the withheld job if the test hook armed one (it arms the next
/// such launch only).
TmaCtl bounded_ctl() {
  TmaCtl ctl;
  ctl.wait_ns = g_wait_ns.load(std::memory_order_relaxed);
  ctl.withhold_job = g_withhold_job.exchange(UINT32_MAX);
  if (ctl.withhold_job != UINT32_MAX) {
    const uint64_t ns = g_withhold_ns.load();
    if (ns)
      ctl.wait_ns = ns;
  }
  return ctl;
}

/// log2 of the column-block group of k_tma_tile's job order (SYM_B200_TMA_GROUP,
/// 0..6; default 3).
uint32_t tma_group_log2() {
  static const uint32_t lg = [] {
    const char *v = std::getenv("SYM_B200_TMA_GROUP");
    const int x = v ? std::atoi(v) : 3;
    return static_cast<uint32_t>(x < 0 ? 0 : x > 6 ? 6 : x);
  }();
  return lg;
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    else
      cudaGetLastError();
  });
  return fn;
}

/// The 3-D view of a [rows, cols] box of `ws`-byte cells used by k_tma_tile:
/// x = column (128 bytes of cells per box), y = group of `gr` rows (stride
/// gr*pitch), z = row in group (stride pitch); box (128 / ws) x (64 / gr) x gr
/// (64 rows) with the 128-byte swizzle. False when the driver rejects the
/// description (the caller then uses a SIMT tile kernel).
bool encode_rows3d(CUtensorMap *map, const void *base, int ws, int64_t cols, int64_t rows, int64_t pitch, int gr,
                   int tile_rows = 64) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
  if (!enc || reinterpret_cast<uintptr_t>(base) % 16 || pitch % 16 || rows % gr || (ws != 1 && ws != 4) ||
      (gr != 4 && gr != 8) || (tile_rows != 64 && tile_rows != 128))
    return false;
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows / gr),
                              static_cast<cuuint64_t>(gr)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(pitch * gr), static_cast<cuuint64_t>(pitch)};
  const cuuint32_t box[3] = {static_cast<cuuint32_t>(128 / ws), static_cast<cuuint32_t>(tile_rows / gr),
                             static_cast<cuuint32_t>(gr)};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = enc(map, ws == 1 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_UINT32, 3,
                         const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <int WS, int WD, int CH> struct TileLaunch {
  static int run(const sbc_relocate &d, int ch_on, int64_t tiles_b, int64_t tiles, int64_t nbatch, cudaStream_t s) {
    if constexpr (WS == 8 || WD == 8) {
      return SBC_EUNSUPPORTED;
    } else {
      const int64_t jobs = tiles * nbatch;
      const int64_t cap = static_cast<int64_t>(sm_count()) * 64;
      const unsigned blocks = static_cast<unsigned>(jobs < cap ? jobs : cap);
      constexpr bool PER_CHANNEL = !(CH == CH_COPY || CH == CH_F16 || CH == CH_BF16 || CH == CH_W16 || CH == CH_WB16);
      if (ch_on == 0 || !PER_CHANNEL)
        k_tile<WS, WD, CH, 0><<<blocks, 256, 0, s>>>(d, tiles_b, tiles, nbatch);
      else if constexpr (PER_CHANNEL) {
        if (ch_on == 1)
          k_tile<WS, WD, CH, 1><<<blocks, 256, 0, s>>>(d, tiles_b, tiles, nbatch);
        else
          k_tile<WS, WD, CH, 2><<<blocks, 256, 0, s>>>(d, tiles_b, tiles, nbatch);
      }
      return launched(cudaSuccess);
    }
  }
};

/// The vectorized tile kernel applies when no axis is padded, every
/// per-channel stage reads one of the two transposed coordinates directly,
/// and both ends keep 16-byte alignment for every tile. Returns the channel
/// axis code (0 none, 1 A, 2 B) or -1.
int tile_eligible(const sbc_relocate &d) {
  const int r = d.rank, ax_a = r - 2, ax_b = r - 1;
  const int ws = d.src_width, wd = d.dst_width;
  if (!((ws == 1 || ws == 2 || ws == 4) && (wd == 1 || wd == 2 || wd == 4)))
    return -1;
  for (int k = 0; k < r; ++k)
    if (d.pad_lo[k] != 0 || d.box_hi[k] > d.extents[k])
      return -1;
  int ch_on = 0;
  for (int k = 0; k < d.nstages; ++k) {
    const sbc_stage &s = d.stages[k];
    if (s.channel == SBC_CH_NONE)
      continue;
    if (s.channel != SBC_CH_AXIS || s.ch_div != 1 || s.ch_mod != 0 || (s.ch_axis != ax_a && s.ch_axis != ax_b))
      return -1;
    const int on = s.ch_axis == ax_a ? 1 : 2;
    if (ch_on && ch_on != on)
      return -1;
    ch_on = on;
  }
  const int64_t Sb = d.src_strides[ax_b], Da = d.dst_strides[ax_a];
  if ((Sb * ws) % 16 || (Da * wd) % 16)
    return -1;
  int64_t si = d.box_lo[ax_a] + d.box_lo[ax_b] * Sb - d.src_offset;
  int64_t di = d.box_lo[ax_a] * Da + d.box_lo[ax_b] - d.dst_offset;
  if (r == 3) {
    if ((d.src_strides[0] * ws) % 16 || (d.dst_strides[0] * wd) % 16)
      return -1;
    si += d.box_lo[0] * d.src_strides[0];
    di += d.box_lo[0] * d.dst_strides[0];
  }
  if ((reinterpret_cast<uintptr_t>(d.src) + si * ws) % 16 || (reinterpret_cast<uintptr_t>(d.dst) + di * wd) % 16)
    return -1;
  return ch_on;
}

bool basic_ok(const sbc_relocate &d) {
  if (d.rank < 1 || d.rank > SBC_MAX_RANK || d.nstages < 0 || d.nstages > SBC_MAX_STAGES || !d.dst)
    return false;
  for (int k = 0; k < d.rank; ++k)
    if (d.box_hi[k] < d.box_lo[k] || d.box_lo[k] < 0 || d.extents[k] < 1)
      return false;
  return true;
}

// Widest warp span of k_narrow (items per lane). Measured on C2 (f32 NCHW
// [64,3,224,224] -> f16 NHWC, pad 3 -> 4): one item per thread 17.4 us,
// residency-capped spans of 2 14.3-15.4 us, spans of 4 (89 registers,
// 2 blocks per SM) 16.4-17.3 us.
#ifndef SBC_NARROW_VMAX
#define SBC_NARROW_VMAX 2
#endif
// SBC_NARROW_BALANCED = 1: size the span grid so every warp takes the same
// number of spans instead of filling every resident slot.
#ifndef SBC_NARROW_BALANCED
#define SBC_NARROW_BALANCED 0
#endif
// SBC_NARROW_CAP = 0: one span per warp (the hardware block scheduler hands
// out the spans) instead of a grid capped at what stays resident. Measured
// on C2: capped 14.34 / 14.34 us, uncapped 14.34 / 14.83 us.
#ifndef SBC_NARROW_CAP
#define SBC_NARROW_CAP 1
#endif


template <int WS, int WD, int CH>
int launch_narrow(const sbc_relocate &d, int nb, int64_t per_batch, int64_t total, cudaStream_t s) {
  const FastDiv pb = make_fastdiv(static_cast<uint32_t>(per_batch));
  const uint32_t n = static_cast<uint32_t>(total);
  // Warp spans of 32 x V items when a batch holds whole spans (all of a
  // lane's loads first; the grid is what stays resident, warps loop over
  // spans); otherwise one item per thread.
  constexpr int VMAX = SBC_NARROW_VMAX;
  const int v = VMAX >= 4 && per_batch % 128 == 0 ? 4 : VMAX >= 2 && per_batch % 64 == 0 ? 2 : 1;
  auto grid = [&](auto kernel) -> unsigned {
    if (v == 1)
      return static_cast<unsigned>((total + 255) / 256);
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, 256, 0) != cudaSuccess || per_sm < 1)
      per_sm = 1;
    const int64_t spans = total / (32 * v), cap = static_cast<int64_t>(sm_count()) * per_sm;
#if SBC_NARROW_BALANCED
    // As many rounds of spans as the resident grid needs, then just enough
    // warps that every warp takes that many: no last round with a third of
    // the warps idle.
    const int64_t rounds = (spans + cap * 8 - 1) / (cap * 8);
    const int64_t warps = (spans + rounds - 1) / rounds;
    return static_cast<unsigned>((warps + 7) / 8);
#else
    const int64_t want = (spans + 7) / 8;
    return static_cast<unsigned>(SBC_NARROW_CAP && want > cap ? cap : want);
#endif
  };
#define SBC_NARROW(NB_, V_)                                                                                  \
  k_narrow<WS, WD, CH, NB_, V_><<<grid(k_narrow<WS, WD, CH, NB_, V_>), 256, 0, s>>>(d, pb, n)
#define SBC_NARROW_V(NB_)                                                                                    \
  (v == 4 ? SBC_NARROW(NB_, 4) : v == 2 ? SBC_NARROW(NB_, 2) : SBC_NARROW(NB_, 1))
  switch (nb) {
  case 2: SBC_NARROW_V(2); break;
  case 3: SBC_NARROW_V(3); break;
  default: SBC_NARROW_V(4); break;
  }
#undef SBC_NARROW_V
#undef SBC_NARROW
  return launched(cudaSuccess);
}

template <int WS, int WD, int CH> struct RunsLaunch {
  static int run(const sbc_relocate &d, const RunsGeom &g, uint32_t nunits, cudaStream_t s) {
    if constexpr (WS == 8 || WD == 8 || CH == CH_ANY) {
      return SBC_EUNSUPPORTED;
    } else {
      const uint32_t upr = g.upr.d;
      if (upr % 128 == 0) { // spans of 32 x 4 units inside a row
        const int64_t blocks = grid_for(nunits / 128 * 32, 256, 8);
        k_runs<WS, WD, CH, 4><<<static_cast<unsigned>(blocks), 256, 0, s>>>(d, g, nunits);
      } else if (upr % 64 == 0) {
        const int64_t blocks = grid_for(nunits / 64 * 32, 256, 8);
        k_runs<WS, WD, CH, 2><<<static_cast<unsigned>(blocks), 256, 0, s>>>(d, g, nunits);
      } else {
        const int64_t blocks = grid_for(nunits, 256, 8);
        k_runs<WS, WD, CH, 1><<<static_cast<unsigned>(blocks), 256, 0, s>>>(d, g, nunits);
      }
      return launched(cudaSuccess);
    }
  }
};

/// k_narrow when the box fits it (see the kernel); SBC_EUNSUPPORTED otherwise.
int try_narrow(const sbc_relocate &d, int chain, cudaStream_t s) {
  const int ax_a = d.rank - 2, ax_b = d.rank - 1;
  const int64_t ext_a = d.box_hi[ax_a] - d.box_lo[ax_a], nb = d.box_hi[ax_b] - d.box_lo[ax_b];
  const int ws = d.src_width, wd = d.dst_width;
  if (nb < 2 || nb > 4 || ws < 2 || d.dst_strides[ax_a] != nb)
    return SBC_EUNSUPPORTED;
  if (chain == CH_Q || chain == CH_DQ) {
    if (d.stages[0].channel != SBC_CH_NONE || d.stages[0].channel_length < 1)
      return SBC_EUNSUPPORTED;
  } else if (chain != CH_COPY && chain != CH_F16 && chain != CH_BF16 && chain != CH_W16 && chain != CH_WB16) {
    return SBC_EUNSUPPORTED;
  }
  const int va = 16 / ws;
  const int run = va * static_cast<int>(nb) * wd;
  const int sv = run % 16 == 0 ? 16 : run % 8 == 0 ? 8 : 4;
  if (ext_a % va || run % 4)
    return SBC_EUNSUPPORTED;
  // every A (and batch) cell of the box is a valid source cell
  for (int k = 0; k <= ax_a; ++k)
    if (d.box_lo[k] < d.pad_lo[k] || d.box_hi[k] > d.pad_lo[k] + d.extents[k])
      return SBC_EUNSUPPORTED;
  int64_t s0 = d.box_lo[ax_a] - d.pad_lo[ax_a] - d.src_offset;
  int64_t d0 = d.box_lo[ax_a] * nb + d.box_lo[ax_b] - d.dst_offset;
  if (d.rank == 3) {
    s0 += (d.box_lo[0] - d.pad_lo[0]) * d.src_strides[0];
    d0 += d.box_lo[0] * d.dst_strides[0];
    if ((d.src_strides[0] * ws) % 16 || (d.dst_strides[0] * wd) % sv)
      return SBC_EUNSUPPORTED;
  }
  if ((reinterpret_cast<uintptr_t>(d.src) + s0 * ws) % 16 || (d.src_strides[ax_b] * ws) % 16 ||
      (reinterpret_cast<uintptr_t>(d.dst) + d0 * wd) % sv)
    return SBC_EUNSUPPORTED;
  const int64_t per_batch = ext_a / va;
  const int64_t total = per_batch * (d.rank == 3 ? d.box_hi[0] - d.box_lo[0] : 1);
  if (total >= (int64_t(1) << 31) - 256 * 8 * 1024) // 32-bit thread indices, grid stride included
    return SBC_EUNSUPPORTED;
  const int n = static_cast<int>(nb);
  if (chain == CH_COPY && ws == 4 && wd == 4)
    return launch_narrow<4, 4, CH_COPY>(d, n, per_batch, total, s);
  if (chain == CH_COPY && ws == 2 && wd == 2)
    return launch_narrow<2, 2, CH_COPY>(d, n, per_batch, total, s);
  if (chain == CH_F16 && ws == 4 && wd == 2)
    return launch_narrow<4, 2, CH_F16>(d, n, per_batch, total, s);
  if (chain == CH_BF16 && ws == 4 && wd == 2)
    return launch_narrow<4, 2, CH_BF16>(d, n, per_batch, total, s);
  if (chain == CH_W16 && ws == 2 && wd == 4)
    return launch_narrow<2, 4, CH_W16>(d, n, per_batch, total, s);
  if (chain == CH_WB16 && ws == 2 && wd == 4)
    return launch_narrow<2, 4, CH_WB16>(d, n, per_batch, total, s);
  if (chain == CH_Q && ws == 4 && wd == 1)
    return launch_narrow<4, 1, CH_Q>(d, n, per_batch, total, s);
  return SBC_EUNSUPPORTED;
}

int64_t box_count(const sbc_relocate &d) {
  int64_t n = 1;
  for (int k = 0; k < d.rank; ++k)
    n *= d.box_hi[k] - d.box_lo[k];
  return n;
}

/// The TMA tile kernel over `n` sources: source j starts at `bases[j]` and
/// holds `rows[j]` consecutive rows of axis B (the source-row axis), in
/// order, together the box's whole B extent. SBC_EUNSUPPORTED when the box or
/// a source does not fit the kernel (the caller uses another kernel).
int launch_tma(const sbc_relocate &d, int chain, int ch_on, const void *const *bases, const int64_t *rows, int n,
               cudaStream_t st) {
  if (d.rank != 2 || n < 1 || n > kMaxTmaSources || !tma_enabled())
    return SBC_EUNSUPPORTED;
  const int64_t ext_a = d.box_hi[0] - d.box_lo[0], ext_b = d.box_hi[1] - d.box_lo[1];
  const bool tma_s8 = d.src_width == 1 && d.dst_width == 2 && (chain == CH_DQ_F16 || chain == CH_DQ_BF16);
  const bool tma_32 = d.src_width == 4 && ch_on == 0 &&
                      ((chain == CH_COPY && d.dst_width == 4) ||
                       ((chain == CH_F16 || chain == CH_BF16) && d.dst_width == 2));
  const int64_t tma_ta = 128 / d.src_width;
  if (ch_on < 0 || !(tma_s8 || tma_32) || ext_a % tma_ta || ext_b % 64 ||
      (ext_a / tma_ta) * (ext_b / 64) >= (int64_t(1) << 31))
    return SBC_EUNSUPPORTED;
  const int group = tma_32 && chain == CH_COPY ? 4 : 8; // rows per view group, as the kernel's GR
  // int8 sources whose blocks are all whole 128-row tiles take the tall tile
  bool tall = tma_s8 && tma_tall_enabled() && ext_b % 128 == 0;
  for (int j = 0; j < n && tall; ++j)
    tall = rows[j] > 0 && rows[j] % 128 == 0;
  const int64_t tb_rows = tall ? 128 : 64;
  TmaSources srcs{};
  srcs.n = n;
  int64_t covered = 0;
  for (int j = 0; j < n; ++j) {
    if (rows[j] <= 0 || rows[j] % 64)
      return SBC_EUNSUPPORTED;
    srcs.tb_first[j] = static_cast<uint32_t>(covered / tb_rows);
    if (!encode_rows3d(&srcs.map[j], bases[j], d.src_width, ext_a, rows[j], d.src_strides[1] * d.src_width,
                       group, static_cast<int>(tb_rows)))
      return SBC_EUNSUPPORTED;
    covered += rows[j];
  }
  if (covered != ext_b)
    return SBC_EUNSUPPORTED;
  const int64_t tiles_b = ext_b / tb_rows, tiles = (ext_a / tma_ta) * tiles_b;
  srcs.tb_first[n] = static_cast<uint32_t>(tiles_b);
  const int64_t cap = static_cast<int64_t>(sm_count()) * SBC_TMA_CTAS_PER_SM;
  const unsigned blocks = static_cast<unsigned>(tiles < cap ? tiles : cap);
  TileOrder ord;
  ord.lg = tma_group_log2();
  while (ord.lg > 0 && (ext_a / tma_ta) % (int64_t(1) << ord.lg))
    --ord.lg;
  ord.group = make_fastdiv(static_cast<uint32_t>(tiles_b << ord.lg));
  const size_t smem = (tall ? KTallStages * KTallTileBytes : KStages * KTmaTileBytes) + 1024;
  const uint32_t nt = static_cast<uint32_t>(tiles);
  const TmaCtl ctl = bounded_ctl();
#define SBC_TMA(WS_, CH_, ON_)                                                                                 \
  (cudaFuncSetAttribute(k_tma_tile<WS_, CH_, ON_>, cudaFuncAttributeMaxDynamicSharedMemorySize,                    \
                        static_cast<int>(smem)),                                                                 \
   k_tma_tile<WS_, CH_, ON_><<<blocks, KTmaThreads, smem, st>>>(srcs, d, ord, nt, ctl))
  const bool dynamic = tall && tma_dynamic_enabled();
#define SBC_TALL_(CH_, ON_, DYN_, GRID_)                                                                       \
  (cudaFuncSetAttribute(k_tma_tall<CH_, ON_, DYN_>, cudaFuncAttributeMaxDynamicSharedMemorySize,                  \
                        static_cast<int>(smem)),                                                                 \
   k_tma_tall<CH_, ON_, DYN_><<<GRID_, KTmaThreads, smem, st>>>(srcs, d, ord, nt, ctl))
#define SBC_TALL(CH_, ON_) (dynamic ? SBC_TALL_(CH_, ON_, true, nt) : SBC_TALL_(CH_, ON_, false, blocks))
  if (tall && chain == CH_DQ_F16)
    ch_on == 0 ? SBC_TALL(CH_DQ_F16, 0) : ch_on == 1 ? SBC_TALL(CH_DQ_F16, 1) : SBC_TALL(CH_DQ_F16, 2);
  else if (tall)
    ch_on == 0 ? SBC_TALL(CH_DQ_BF16, 0) : ch_on == 1 ? SBC_TALL(CH_DQ_BF16, 1) : SBC_TALL(CH_DQ_BF16, 2);
  else if (tma_32)
    chain == CH_COPY ? SBC_TMA(4, CH_COPY, 0) : chain == CH_F16 ? SBC_TMA(4, CH_F16, 0) : SBC_TMA(4, CH_BF16, 0);
  else if (chain == CH_DQ_F16)
    ch_on == 0 ? SBC_TMA(1, CH_DQ_F16, 0) : ch_on == 1 ? SBC_TMA(1, CH_DQ_F16, 1) : SBC_TMA(1, CH_DQ_F16, 2);
  else
    ch_on == 0 ? SBC_TMA(1, CH_DQ_BF16, 0) : ch_on == 1 ? SBC_TMA(1, CH_DQ_BF16, 1) : SBC_TMA(1, CH_DQ_BF16, 2);
#undef SBC_TALL
#undef SBC_TALL_
#undef SBC_TMA
  g_wait_launches.fetch_add(1, std::memory_order_relaxed);
  return launched(cudaSuccess);
}

} // namespace

extern "C" {

int sbc_relocate_transpose_shards(const sbc_relocate *desc, const void *const *srcs, const int64_t *row_bounds,
                                  int32_t n, void *stream) {
  if (!desc || !basic_ok(*desc) || !srcs || !row_bounds || n < 1)
    return SBC_EINVAL;
  const sbc_relocate &d = *desc;
  if (d.rank != 2 || d.src_strides[0] != 1 || d.dst_strides[1] != 1 || n > kMaxTmaSources)
    return SBC_EUNSUPPORTED;
  const int chain = chain_of(d);
  if (!chain_channels_ok(d, chain, true))
    return SBC_EUNSUPPORTED;
  // the shards tile the box's source rows exactly
  if (row_bounds[0] != d.box_lo[1] - d.pad_lo[1] || row_bounds[n] != d.box_hi[1] - d.pad_lo[1])
    return SBC_EUNSUPPORTED;
  int64_t rows[kMaxTmaSources];
  for (int j = 0; j < n; ++j)
    rows[j] = row_bounds[j + 1] - row_bounds[j];
  // the eligibility checks see the first block as the source
  sbc_relocate e = d;
  e.src = srcs[0];
  e.src_offset = row_bounds[0] * d.src_strides[1];
  return launch_tma(e, chain, tile_eligible(e), srcs, rows, n, static_cast<cudaStream_t>(stream));
}

int sbc_relocate_generic(const sbc_relocate *desc, void *stream) {
  if (!desc || !basic_ok(*desc))
    return SBC_EINVAL;
  const int64_t total = box_count(*desc);
  if (total == 0)
    return 0;
  int chain = chain_of(*desc);
  if (!chain_channels_ok(*desc, chain, true))
    chain = CH_ANY;
  if (desc->src_width == 8 || desc->dst_width == 8)
    chain = desc->nstages == 0 && desc->src_width == desc->dst_width ? CH_COPY : -1;
  return dispatch<GenericLaunch>(desc->src_width, desc->dst_width, chain, *desc, total,
                                 static_cast<cudaStream_t>(stream));
}

int sbc_relocate_runs(const sbc_relocate *desc, void *stream) {
  if (!desc || !basic_ok(*desc))
    return SBC_EINVAL;
  const sbc_relocate &d = *desc;
  const int r = d.rank, last = r - 1;
  if (r < 2 || d.src_strides[last] != 1 || d.dst_strides[last] != 1 || d.src_width == 8 || d.dst_width == 8)
    return SBC_EUNSUPPORTED;
  const int chain = chain_of(d);
  if (chain == CH_ANY)
    return SBC_EUNSUPPORTED;
  if (chain == CH_Q || chain == CH_DQ || chain == CH_DQ_F16 || chain == CH_DQ_BF16) {
    const sbc_stage &s = d.stages[0];
    const bool outer_axis = s.channel == SBC_CH_AXIS && s.ch_axis < last && s.ch_div >= 1 && s.ch_mod >= 0;
    if ((s.channel != SBC_CH_NONE && !outer_axis) || s.channel_length < 1)
      return SBC_EUNSUPPORTED;
  }
  const int ws = d.src_width, wd = d.dst_width;
  const int U = 16 / (ws > wd ? ws : wd);
  // the last axis of the box lies in the valid source and splits into units
  const int64_t run = d.box_hi[last] - d.box_lo[last];
  if (d.box_lo[last] < d.pad_lo[last] || d.box_hi[last] > d.pad_lo[last] + d.extents[last] || run % U)
    return SBC_EUNSUPPORTED;
  int64_t rows = 1;
  for (int k = 0; k < last; ++k) {
    const int64_t e = d.box_hi[k] - d.box_lo[k];
    if (d.src_strides[k] % U || d.dst_strides[k] % U || e >= (int64_t(1) << 31))
      return SBC_EUNSUPPORTED;
    rows *= e;
  }
  if (run == 0 || rows == 0)
    return 0;
  const int64_t upr = run / U, nunits = rows * upr;
  if (upr >= (int64_t(1) << 31) || nunits >= (int64_t(1) << 31) - 256 * 8 * 1024) // 32-bit unit indices
    return SBC_EUNSUPPORTED;
  // every unit starts 16-byte aligned on the wide side (and U-element aligned on the other)
  const uintptr_t sa = reinterpret_cast<uintptr_t>(d.src) + (d.box_lo[last] - d.pad_lo[last] - d.src_offset) * ws;
  const uintptr_t da = reinterpret_cast<uintptr_t>(d.dst) + (d.box_lo[last] - d.dst_offset) * wd;
  if (sa % (U * ws) || da % (U * wd))
    return SBC_EUNSUPPORTED;
  RunsGeom g;
  g.upr = make_fastdiv(static_cast<uint32_t>(upr));
  for (int k = 0; k < SBC_MAX_RANK - 1; ++k)
    g.ext[k] = make_fastdiv(k < last ? static_cast<uint32_t>(d.box_hi[k] - d.box_lo[k]) : 1u);
  return dispatch<RunsLaunch>(ws, wd, chain, d, g, static_cast<uint32_t>(nunits), static_cast<cudaStream_t>(stream));
}

int sbc_relocate_contiguous(const sbc_relocate *desc, void *stream) {
  if (!desc || !basic_ok(*desc))
    return SBC_EINVAL;
  const sbc_relocate &d = *desc;
  if (d.rank != 1 || d.src_strides[0] != 1 || d.dst_strides[0] != 1)
    return SBC_EUNSUPPORTED;
  int chain = chain_of(d);
  if (!chain_channels_ok(d, chain, false))
    return SBC_EUNSUPPORTED;
  const int ws = d.src_width, wd = d.dst_width;
  if (ws == 8 || wd == 8)
    return SBC_EUNSUPPORTED;
  const int minw = ws < wd ? ws : wd, maxw = ws < wd ? wd : ws;
  const int V = 16 / minw, U = 16 / maxw; // alignment period; elements per kernel unit
  // Valid part of the box, then its 16-byte aligned body of whole units.
  const int64_t lo = d.box_lo[0], hi = d.box_hi[0];
  const int64_t v0 = lo > d.pad_lo[0] ? lo : d.pad_lo[0];
  const int64_t vend = d.pad_lo[0] + d.extents[0];
  const int64_t v1 = hi < vend ? hi : vend;
  int64_t body0 = v0, nunits = 0;
  if (v1 > v0) {
    const uintptr_t sa = reinterpret_cast<uintptr_t>(d.src) + (v0 - d.pad_lo[0] - d.src_offset) * ws;
    const uintptr_t da = reinterpret_cast<uintptr_t>(d.dst) + (v0 - d.dst_offset) * wd;
    // advance to the first element where both addresses are 16-byte aligned
    int64_t skip = -1;
    for (int64_t i = 0; i < V && v0 + i < v1; ++i)
      if ((sa + i * ws) % 16 == 0 && (da + i * wd) % 16 == 0) {
        skip = i;
        break;
      }
    if (skip >= 0) {
      body0 = v0 + skip;
      nunits = (v1 - body0) / U;
    }
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // Scalar remainder (head, tail, pads) through the generic kernel.
  auto generic_range = [&](int64_t a, int64_t b) -> int {
    if (b <= a)
      return 0;
    sbc_relocate part = d;
    part.box_lo[0] = a;
    part.box_hi[0] = b;
    return sbc_relocate_generic(&part, stream);
  };
  if (nunits == 0)
    return generic_range(lo, hi);
  // A few cells on either side of the body (unaligned ends, a short pad)
  // ride along in the body's launch; longer ends take the generic kernel.
  const int64_t body1 = body0 + nunits * U;
  ScalarEnds ends;
  const bool fold = (body0 - lo) + (hi - body1) <= 4096;
  if (fold) {
    ends.head_lo = lo;
    ends.nhead = static_cast<int32_t>(body0 - lo);
    ends.tail_lo = body1;
    ends.ntail = static_cast<int32_t>(hi - body1);
  }
  int rc = dispatch<ContiguousLaunch>(ws, wd, chain, d, body0, nunits, ends, s);
  if (rc || fold)
    return rc;
  if ((rc = generic_range(lo, body0)))
    return rc;
  return generic_range(body1, hi);
}

int sbc_relocate_transpose(const sbc_relocate *desc, void *stream) {
  if (!desc || !basic_ok(*desc))
    return SBC_EINVAL;
  const sbc_relocate &d = *desc;
  if (d.rank != 2 && d.rank != 3)
    return SBC_EUNSUPPORTED;
  const int ax_a = d.rank - 2, ax_b = d.rank - 1;
  if (d.src_strides[ax_a] != 1 || d.dst_strides[ax_b] != 1)
    return SBC_EUNSUPPORTED;
  int chain = chain_of(d);
  if (!chain_channels_ok(d, chain, true))
    return SBC_EUNSUPPORTED;
  if (d.src_width == 8 || d.dst_width == 8)
    return SBC_EUNSUPPORTED;
  const int64_t ext_a = d.box_hi[ax_a] - d.box_lo[ax_a], ext_b = d.box_hi[ax_b] - d.box_lo[ax_b];
  const int64_t nbatch = d.rank == 3 ? d.box_hi[0] - d.box_lo[0] : 1;
  if (ext_a == 0 || ext_b == 0 || nbatch == 0)
    return 0;
  if (ext_b <= 4) {
    const int rc = try_narrow(d, chain, static_cast<cudaStream_t>(stream));
    if (rc != SBC_EUNSUPPORTED)
      return rc;
  }
  const int ch_on = tile_eligible(d);
  const bool dq = chain == CH_DQ || chain == CH_DQ_F16 || chain == CH_DQ_BF16;
  {
    const void *base = static_cast<const uint8_t *>(d.src) +
                       (d.box_lo[0] + d.box_lo[1] * d.src_strides[1] - d.src_offset) * d.src_width;
    const int rc = launch_tma(d, chain, ch_on, &base, &ext_b, 1, static_cast<cudaStream_t>(stream));
    if (rc != SBC_EUNSUPPORTED)
      return rc;
  }
  if (ch_on >= 0 && dq && d.src_width == 1 && ext_a >= 128 && ext_b * d.dst_width >= 128 &&
      ((ext_a + 127) / 128) * ((ext_b * d.dst_width + 127) / 128) * nbatch < (int64_t(1) << 31)) {
    const int64_t tbn = 128 / d.dst_width;
    const int64_t tiles_b = (ext_b + tbn - 1) / tbn, tiles = ((ext_a + 127) / 128) * tiles_b;
    const int64_t jobs = tiles * nbatch, cap = static_cast<int64_t>(sm_count()) * 8;
    const unsigned blocks = static_cast<unsigned>(jobs < cap ? jobs : cap);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    auto fast = [](uint32_t dv) {
      FastDiv f;
      uint32_t l = 0;
      while ((1ull << l) < dv)
        ++l;
      f.s = 31 + l;
      f.d = dv;
      f.m = ((1ull << f.s) + dv - 1) / dv;
      return f;
    };
    const FastDiv div_b = fast(static_cast<uint32_t>(tiles_b)), div_t = fast(static_cast<uint32_t>(tiles));
#define SBC_S8(WD_, CH_, ON_)                                                                                  \
  k_tile_s8<WD_, CH_, ON_><<<blocks, 256, 0, s>>>(d, div_b, div_t, static_cast<uint32_t>(jobs))
#define SBC_S8_ON(WD_, CH_)                                                                                     \
  do {                                                                                                         \
    if (ch_on == 0)                                                                                            \
      SBC_S8(WD_, CH_, 0);                                                                                     \
    else if (ch_on == 1)                                                                                       \
      SBC_S8(WD_, CH_, 1);                                                                                     \
    else                                                                                                       \
      SBC_S8(WD_, CH_, 2);                                                                                     \
  } while (0)
    if (chain == CH_DQ_F16 && d.dst_width == 2)
      SBC_S8_ON(2, CH_DQ_F16);
    else if (chain == CH_DQ_BF16 && d.dst_width == 2)
      SBC_S8_ON(2, CH_DQ_BF16);
    else if (chain == CH_DQ && d.dst_width == 4)
      SBC_S8_ON(4, CH_DQ);
#undef SBC_S8_ON
#undef SBC_S8
    return launched(cudaSuccess);
  }
  if (ch_on >= 0 && ext_a * d.src_width >= 128 && ext_b * d.dst_width >= 128) {
    const int64_t ta = 128 / d.src_width, tbn = 128 / d.dst_width;
    const int64_t tiles_b = (ext_b + tbn - 1) / tbn, tiles = ((ext_a + ta - 1) / ta) * tiles_b;
    const int rc = dispatch<TileLaunch>(d.src_width, d.dst_width, chain, d, ch_on, tiles_b, tiles, nbatch,
                                        static_cast<cudaStream_t>(stream));
    if (rc != SBC_EUNSUPPORTED)
      return rc;
  }
  // Tile shape: a short destination row (B) takes the whole row so the tile
  // is one contiguous destination block; otherwise 64 x 64.
  int tb = 64, ta = 64;
  if (ext_b <= 16) {
    tb = static_cast<int>(ext_b);
    ta = 2048 / tb;
  }
  const int64_t tiles_a = (ext_a + ta - 1) / ta, tiles_b = (ext_b + tb - 1) / tb;
  return dispatch<TransposeLaunch>(d.src_width, d.dst_width, chain, d, ta, tb, tiles_a, tiles_b, nbatch,
                                   static_cast<cudaStream_t>(stream));
}

int sbc_fill(void *dst, int64_t count, int32_t width, uint64_t bits, void *stream) {
  if (count <= 0)
    return 0;
  const int64_t blocks = grid_for(count, 256, 8);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (width) {
  case 1: k_fill<1><<<static_cast<unsigned>(blocks), 256, 0, s>>>(dst, count, bits); break;
  case 2: k_fill<2><<<static_cast<unsigned>(blocks), 256, 0, s>>>(dst, count, bits); break;
  case 4: k_fill<4><<<static_cast<unsigned>(blocks), 256, 0, s>>>(dst, count, bits); break;
  case 8: k_fill<8><<<static_cast<unsigned>(blocks), 256, 0, s>>>(dst, count, bits); break;
  default: return SBC_EINVAL;
  }
  return launched(cudaSuccess);
}

uint64_t sbc_launch_count(void) { return g_launches.load(); }

uint64_t sbc_wait_launch_count(void) { return g_wait_launches.load(); }

void sbc_set_wait_limit_ns(uint64_t ns) { g_wait_ns.store(ns ? ns : kDefaultWaitLimitNs); }

void sbc_test_withhold_tile(uint32_t job, uint64_t wait_limit_ns) {
  g_withhold_ns.store(wait_limit_ns);
  g_withhold_job.store(job);
}

} // extern "C"
