// Lowering of typed programs to the fused sm_100a kernels and the H2D data
// paths. See device_plan.hpp.
//
// Data paths (routes a and b of the design):
//  * DmaRing: the raw source is cut into chunks of whole source rows (the
//    coalesced axis with the largest source stride), each chunk DMA'd by the
//    copy engine into a slot of an HBM ring on the copy stream, and the fused
//    kernel for that chunk's destination box runs on the compute stream as
//    soon as the chunk lands. Slot reuse is gated by events, so PCIe DMA of
//    chunk i+1.. overlaps the kernel of chunk i. A row window on the
//    destination (multi-GPU shards) whose source is a column range of every
//    source row is gathered with one 2-D DMA per chunk.
//  * ZeroCopy: the fused kernel reads mapped pinned host memory directly.
//  * Staged: one DMA of the (windowed) source, then one kernel.
// No route transforms data on the CPU.
#include "device_plan.hpp"

#include <algorithm>
#include <climits>
#include <cstring>

namespace reloc {
namespace b200 {
namespace {

TransferError terr(const char *code, std::string msg) { return TransferError{code, std::move(msg)}; }

bool isF32(ElementType t) { return t.kind == ElementTypeKind::Float && t.bitwidth == 32; }
bool isBF16(ElementType t) { return t.kind == ElementTypeKind::BFloat && t.bitwidth == 16; }

int stageOp(const typed::StageArithmetic &s) {
  switch (s.transform) {
  case ValueTransformKind::Cast:
    if (isF32(s.input))
      return isBF16(s.output) ? SBC_NARROW_BF16 : SBC_NARROW_F16;
    return isBF16(s.input) ? SBC_WIDEN_BF16 : SBC_WIDEN_F16;
  case ValueTransformKind::Quantize:
    return SBC_QUANTIZE;
  case ValueTransformKind::Dequantize:
    return SBC_DEQUANTIZE;
  }
  return SBC_NARROW_F16;
}

constexpr size_t kNone = SIZE_MAX;
constexpr size_t kDefaultChunkBytes = size_t(8) << 20;
constexpr size_t kMaxChunkBytes = size_t(64) << 20;

/// Rows per chunk rounded down to whole tiles: multiples of 128 rows (the
/// tall int8 tiles) when at least 128, else of 64, else unchanged.
int64_t wholeTileRows(int64_t rows) {
  if (rows >= 128)
    return rows - rows % 128;
  if (rows >= 64)
    return rows - rows % 64;
  return rows;
}

} // namespace

namespace {

/// The staging buffer for `bytes` within the context's live scratch budget:
/// ring scratch is released first when both do not fit.
std::variant<void *, TransferError> budgetedStaging(CudaBackend &b, size_t bytes) {
  bytes = bytes ? bytes : 16;
  if (b.liveLimit && bytes > b.stagingCapacity()) {
    if (bytes + 16 > b.liveLimit)
      return terr("insufficient_capacity", "a staging buffer of " + std::to_string(bytes) +
                                               " bytes exceeds the context's live scratch budget of " +
                                               std::to_string(b.liveLimit) + " bytes");
    if (b.deviceBytes() - b.stagingCapacity() + bytes > b.liveLimit)
      b.trim(b.deviceBytes() - b.ringBytes()); // drop the ring, keep the rest
  }
  void *p = b.staging(bytes);
  if (!p)
    return terr("backend_failure", b.error());
  return p;
}

/// The ring-slot size for chunks of `rowBytes`-byte rows: at most `target`,
/// within the live budget (a hard limit: insufficient_capacity when not even
/// one row fits) and, for default chunk sizes, within the retained budget
/// when that still allows default-sized chunks (a smaller retained budget
/// keeps the chunk size, and the ring is released when the lease ends).
std::variant<size_t, TransferError> budgetedChunk(const CudaBackend &b, int slots, size_t target, int64_t rowBytes,
                                                  bool defaultSize) {
  const size_t row = static_cast<size_t>(rowBytes);
  const size_t hard = b.ringSlotBudget(slots, false);
  if (hard < row)
    return terr("insufficient_capacity", "the context's live scratch budget of " + std::to_string(b.liveLimit) +
                                             " bytes holds no ring of " + std::to_string(slots) + " slots of one " +
                                             std::to_string(row) + "-byte row");
  const size_t soft = b.ringSlotBudget(slots, true);
  if (defaultSize && soft >= kDefaultChunkBytes)
    target = std::min(target, soft);
  return std::min(target, hard);
}

} // namespace

const char *familyName(Family f) {
  switch (f) {
  case Family::Contiguous: return "contiguous";
  case Family::Transpose: return "transpose";
  case Family::Runs: return "runs";
  default: return "generic";
  }
}

int launchFamily(Family f, const sbc_relocate &d, void *stream) {
  int rc = SBC_EUNSUPPORTED;
  if (f == Family::Contiguous)
    rc = sbc_relocate_contiguous(&d, stream);
  else if (f == Family::Transpose)
    rc = sbc_relocate_transpose(&d, stream);
  else if (f == Family::Runs)
    rc = sbc_relocate_runs(&d, stream);
  if (rc == SBC_EUNSUPPORTED)
    rc = sbc_relocate_generic(&d, stream);
  return rc;
}

std::variant<Lowered, TransferError> lower(const typed::Program &p) {
  Lowered l;
  sbc_relocate &d = l.desc;
  std::memset(&d, 0, sizeof d);
  const BoundPlan &lay = p.plan.layout;
  const int r = static_cast<int>(lay.extents.size());
  if (r < 1 || r > SBC_MAX_RANK)
    return terr("unsupported_layout", "coalesced rank " + std::to_string(r) + " exceeds the device limit of 8");
  const uint32_t nst = static_cast<uint32_t>(p.stages.size());
  if (nst > SBC_MAX_STAGES)
    return terr("unsupported_stage", "more than 4 value stages");
  auto fill = typed::fillAt(p, nst);
  if (auto *e = std::get_if<typed::ExecutionError>(&fill))
    return terr(e->code.c_str(), e->message);
  const auto &fb = std::get<std::optional<uint64_t>>(fill);
  d.has_fill = fb.has_value();
  d.fill_bits = fb.value_or(0);
  d.rank = r;
  d.src_width = static_cast<int32_t>(typed::widthAt(p, 0));
  d.dst_width = static_cast<int32_t>(typed::widthAt(p, nst));
  for (int k = 0; k < r; ++k) {
    d.extents[k] = lay.extents[k];
    d.src_strides[k] = lay.srcStrides[k];
    d.dst_strides[k] = lay.dstStrides[k];
  }
  for (const PadRegion &pr : lay.padRegions)
    d.pad_lo[pr.axis] = pr.lo;
  int64_t hiPad[SBC_MAX_RANK] = {};
  for (const PadRegion &pr : lay.padRegions)
    hiPad[pr.axis] = pr.hi;
  l.dstElements = 1;
  for (int k = 0; k < r; ++k) {
    l.padded[k] = lay.extents[k] + d.pad_lo[k] + hiPad[k];
    d.box_lo[k] = 0;
    d.box_hi[k] = l.padded[k];
    l.dstElements *= l.padded[k];
  }
  l.srcElements = p.sourceElements;
  // dense row-major destination over the padded box
  {
    int64_t expect = 1;
    l.denseCover = true;
    for (int k = r - 1; k >= 0; --k) {
      if (l.padded[k] != 1 && d.dst_strides[k] != expect)
        l.denseCover = false;
      expect *= l.padded[k];
    }
  }
  const size_t rr = p.plan.resultExtents.size();
  if (rr > SBC_MAX_RANK)
    return terr("unsupported_layout", "result rank exceeds the device limit of 8");
  d.result_rank = static_cast<int32_t>(rr);
  for (size_t j = 0; j < rr; ++j) {
    d.result_extents[j] = p.plan.resultExtents[j];
    d.result_strides[j] = p.resultStrides[j];
  }
  d.nsymbols = static_cast<int32_t>(std::min<size_t>(p.plan.symbols.size(), SBC_MAX_SYMBOLS));
  for (int i = 0; i < d.nsymbols; ++i)
    d.symbols[i] = p.plan.symbols[static_cast<size_t>(i)];

  // Stages and the packed parameter blob (reciprocals for quantize).
  d.nstages = static_cast<int32_t>(nst);
  bool anyExpr = false, anyOffset = false;
  for (uint32_t k = 0; k < nst; ++k) {
    const typed::StageArithmetic &s = p.stages[k];
    sbc_stage &g = d.stages[k];
    g.op = stageOp(s);
    g.channel = SBC_CH_NONE;
    g.channel_length = s.channelLength;
    size_t po = kNone, zo = kNone;
    if (s.transform != ValueTransformKind::Cast) {
      const std::vector<float> &vals = s.transform == ValueTransformKind::Quantize ? s.invScale : s.scale;
      po = l.paramBlob.size();
      l.paramBlob.resize(po + vals.size() * 4);
      std::memcpy(l.paramBlob.data() + po, vals.data(), vals.size() * 4);
      if (s.transform == ValueTransformKind::Dequantize && !s.zeroPoint.empty()) {
        while (l.paramBlob.size() % 4)
          l.paramBlob.push_back(0);
        zo = l.paramBlob.size();
        l.paramBlob.resize(zo + s.zeroPoint.size() * 4);
        std::memcpy(l.paramBlob.data() + zo, s.zeroPoint.data(), s.zeroPoint.size() * 4);
        g.zp_mode = s.zeroPoint.size() == 1 ? 1 : 2;
      }
    }
    l.paramOffset.push_back(po);
    l.zpOffset.push_back(zo);
    if (!s.perChannel)
      continue;
    const ExprStream &ch = p.plan.stages[k].channel;
    if (s.channelIsDim) {
      const uint32_t dim = s.channelDim;
      const int64_t rs = p.resultStrides[dim], re = p.plan.resultExtents[dim];
      bool placed = false;
      if (re == 1) {
        g.channel = SBC_CH_AXIS;
        g.ch_axis = 0;
        g.ch_div = 1;
        g.ch_mod = 1;
        placed = true;
      } else if (l.denseCover) {
        for (int a = 0; a < r && !placed; ++a) {
          const int64_t ds = d.dst_strides[a];
          if (l.padded[a] == 1 || ds > rs || rs % ds != 0 || rs >= ds * l.padded[a])
            continue;
          const int64_t div = rs / ds;
          g.channel = SBC_CH_AXIS;
          g.ch_axis = a;
          g.ch_div = div;
          g.ch_mod = (div * re == l.padded[a]) ? 0 : re;
          placed = true;
        }
      }
      if (!placed) {
        g.channel = SBC_CH_OFFSET;
        g.ch_dim = static_cast<int32_t>(dim);
        anyOffset = true;
      }
      // static range proof: the coordinate never exceeds its extent
      if (re > s.channelLength)
        l.needsStatus = true;
    } else {
      if (ch.size() > SBC_MAX_TOKENS)
        return terr("implementation_unavailable", "channel expression longer than 16 tokens");
      for (const ExprToken &t : ch)
        if (t.op == ExprOp::PushSym && t.value >= SBC_MAX_SYMBOLS)
          return terr("implementation_unavailable", "channel expression uses more than 8 symbols");
      g.channel = SBC_CH_EXPR;
      g.ntokens = static_cast<int32_t>(ch.size());
      for (size_t i = 0; i < ch.size(); ++i) {
        g.token_op[i] = static_cast<int32_t>(ch[i].op);
        g.token_value[i] = ch[i].value;
      }
      anyExpr = true;
      l.needsStatus = true;
    }
  }

  // Kernel family.
  l.family = Family::Generic;
  if (!anyExpr) {
    if (r == 1 && d.src_strides[0] == 1 && d.dst_strides[0] == 1 && !anyOffset)
      l.family = Family::Contiguous;
    else if ((r == 2 || r == 3) && d.src_strides[r - 2] == 1 && d.dst_strides[r - 1] == 1 && l.padded[r - 1] > 1 &&
             l.padded[r - 2] > 1)
      l.family = Family::Transpose;
    else if (r >= 2 && d.src_strides[r - 1] == 1 && d.dst_strides[r - 1] == 1 && l.padded[r - 1] > 1 &&
             !anyOffset)
      l.family = Family::Runs;
  }
  if (d.src_width == 8 || d.dst_width == 8)
    l.family = Family::Generic;

  // Source rows: the axis with the largest source stride, if the source is
  // dense and that axis is outermost (each row is one contiguous block).
  int64_t best = -1;
  for (int k = 0; k < r; ++k)
    if (lay.extents[k] > 1 && d.src_strides[k] > best) {
      best = d.src_strides[k];
      l.srcOuter = k;
    }
  if (l.srcOuter >= 0) {
    const int o = l.srcOuter;
    int64_t span = 0;
    for (int k = 0; k < r; ++k)
      if (k != o)
        span += (lay.extents[k] - 1) * d.src_strides[k];
    l.rowsChunkable = d.src_strides[o] * lay.extents[o] == l.srcElements && span < d.src_strides[o];
  }
  l.classKey = std::string(familyName(l.family)) + ":" + std::to_string(d.src_width) + ">" +
               std::to_string(d.dst_width) + ":" + std::to_string(nst) + ":" +
               std::to_string(64 - __builtin_clzll(static_cast<unsigned long long>(l.srcElements * d.src_width) | 1));
  return l;
}

ParamCache::~ParamCache() {
  int current = -1;
  sbc_get_device(&current);
  for (auto &kv : device) {
    sbc_set_device(kv.first);
    sbc_free_device(kv.second);
  }
  if (current >= 0)
    sbc_set_device(current);
}

std::optional<TransferError> uploadParams(const Lowered &l, CudaBackend &b, sbc_relocate &d) {
  if (l.paramBlob.empty())
    return std::nullopt;
  uint8_t *base = nullptr;
  {
    std::lock_guard<std::mutex> g(l.params->mutex);
    auto it = l.params->device.find(b.device());
    if (it != l.params->device.end()) {
      base = static_cast<uint8_t *>(it->second);
    } else {
      void *p = nullptr;
      int rc = sbc_malloc_device(&p, l.paramBlob.size());
      if (rc) {
        b.fail("cudaMalloc(parameters)", rc);
        return terr("backend_failure", b.error());
      }
      // First use on this device: one blocking upload, then reused.
      if ((rc = sbc_memcpy_h2d_async(p, l.paramBlob.data(), l.paramBlob.size(), b.computeStream())) ||
          (rc = sbc_stream_synchronize(b.computeStream()))) {
        sbc_free_device(p);
        b.fail("parameter upload", rc);
        return terr("backend_failure", b.error());
      }
      ++b.copyCalls;
      l.params->device[b.device()] = p;
      base = static_cast<uint8_t *>(p);
    }
  }
  for (int k = 0; k < d.nstages; ++k) {
    if (l.paramOffset[static_cast<size_t>(k)] != kNone)
      d.stages[k].param = reinterpret_cast<const float *>(base + l.paramOffset[static_cast<size_t>(k)]);
    if (l.zpOffset[static_cast<size_t>(k)] != kNone)
      d.stages[k].zero_point = reinterpret_cast<const int32_t *>(base + l.zpOffset[static_cast<size_t>(k)]);
  }
  return std::nullopt;
}

namespace {

/// Launch the family kernel for `d` on the compute stream, with this
/// context's fault word.
std::optional<TransferError> launch(const Lowered &l, CudaBackend &b, const sbc_relocate &d, RunStats &st) {
  sbc_relocate e = d;
  e.fault = b.faultWord();
  const int rc = launchFamily(l.family, e, b.computeStream());
  if (rc) {
    b.fail("relocation kernel", rc);
    return terr("backend_failure", b.error());
  }
  ++st.launches;
  ++b.kernelLaunches;
  return std::nullopt;
}

/// Apply the row window to the descriptor's axis-0 box and destination rebase.
bool applyWindow(const Lowered &l, sbc_relocate &d, RowWindow w) {
  const int64_t end = w.end < 0 ? l.padded[0] : w.end;
  if (w.begin < 0 || end > l.padded[0] || end < w.begin)
    return false;
  d.box_lo[0] = w.begin;
  d.box_hi[0] = end;
  d.dst_offset = w.begin * d.dst_strides[0];
  return true;
}

bool isWhole(const Lowered &l, RowWindow w) { return w.begin == 0 && (w.end < 0 || w.end == l.padded[0]); }

std::optional<TransferError> prefill(const Lowered &l, CudaBackend &b, void *ddst, RowWindow w, RunStats &st) {
  // Gather kernels write exactly the box; a destination the box does not
  // cover densely gets the fill first (the reference fills, then walks).
  if (!l.desc.has_fill || l.denseCover || !isWhole(l, w))
    return std::nullopt;
  const int rc = sbc_fill(ddst, l.dstElements, l.desc.dst_width, l.desc.fill_bits, b.computeStream());
  if (rc) {
    b.fail("fill kernel", rc);
    return terr("backend_failure", b.error());
  }
  ++st.launches;
  ++b.kernelLaunches;
  return std::nullopt;
}

std::optional<TransferError> zeroStatus(const Lowered &l, CudaBackend &b, sbc_relocate &d) {
  if (!l.needsStatus)
    return std::nullopt;
  d.status = b.statusWord();
  if (b.keepStatus) // a group cleared it before its first member
    return std::nullopt;
  const int rc = sbc_fill(b.statusWord(), 1, 4, 0, b.computeStream());
  if (rc) {
    b.fail("status reset", rc);
    return terr("backend_failure", b.error());
  }
  return std::nullopt;
}

} // namespace

std::optional<TransferError> runDevice(const Lowered &l, CudaBackend &b, const void *dsrc, void *ddst, RowWindow w,
                                       RunStats &st) {
  sbc_relocate d = l.desc;
  if (!applyWindow(l, d, w))
    return terr("invalid_options", "row window outside the padded result");
  if (auto e = uploadParams(l, b, d))
    return e;
  if (auto e = zeroStatus(l, b, d))
    return e;
  if (auto e = prefill(l, b, ddst, w, st))
    return e;
  d.src = dsrc;
  d.dst = ddst;
  st.kernel = familyName(l.family);
  return launch(l, b, d, st);
}

namespace {

/// Rows of axis 0 are contiguous slabs of the destination (the box covers a
/// dense destination and axis 0 is its outermost axis).
bool d2hRows(const Lowered &l) {
  return l.denseCover && l.desc.dst_strides[0] * l.padded[0] == l.dstElements && l.padded[0] > 1;
}

bool mappedPinned(void *host, void **mapped) {
  int kind = 0, dev = -1;
  return sbc_pointer_info(host, &kind, &dev) == 0 && kind == 1 && sbc_host_device_pointer(host, mapped) == 0;
}

} // namespace

Route chooseRouteD2H(const Lowered &l, void *hdst, const TransferOptions &o) {
  if (o.route != Route::Auto)
    return o.route;
  void *mapped = nullptr;
  if (d2hRows(l))
    return Route::DmaRing;
  return mappedPinned(hdst, &mapped) ? Route::ZeroCopy : Route::Staged;
}

std::optional<TransferError> runD2H(const Lowered &l, CudaBackend &b, const void *dsrc, void *hdst, Route route,
                                    const TransferOptions &o, RunStats &st) {
  const int wd = l.desc.dst_width;
  const int64_t dstBytes = l.dstElements * wd;
  if (route == Route::ZeroCopy) {
    void *mapped = nullptr;
    if (!mappedPinned(hdst, &mapped))
      return terr("invalid_view", "zero_copy needs a mapped pinned host destination");
    st.route = "zero_copy";
    st.payloadBytes += dstBytes;
    return runDevice(l, b, dsrc, mapped, RowWindow{}, st);
  }
  // Chunks of whole result rows through the ring; else the whole result
  // through the staging buffer.
  const bool rows = route != Route::Staged && d2hRows(l);
  const int64_t rowBytes = rows ? l.desc.dst_strides[0] * wd : std::max<int64_t>(dstBytes, 1);
  const int64_t nrows = rows ? l.padded[0] : 1;
  const int slots = rows ? std::max(2, o.nBuffers) : 1;
  size_t target = o.chunkSizeOverride ? o.chunkSizeOverride : kDefaultChunkBytes;
  if (rows) {
    auto t = budgetedChunk(b, slots, target, rowBytes, !o.chunkSizeOverride);
    if (auto *e = std::get_if<TransferError>(&t))
      return *e;
    target = std::get<size_t>(t);
  }
  int64_t rowsPer = rows ? std::max<int64_t>(1, static_cast<int64_t>(target) / rowBytes) : 1;
  if (rowsPer >= 64)
    rowsPer -= rowsPer % 64; // whole kernel tiles per chunk
  void *stage = nullptr;
  if (rows) {
    if (!b.ensureRing(slots, static_cast<size_t>(rowsPer * rowBytes)))
      return terr("backend_failure", b.error());
  } else {
    auto sg = budgetedStaging(b, static_cast<size_t>(rowBytes));
    if (auto *e = std::get_if<TransferError>(&sg))
      return *e;
    stage = std::get<void *>(sg);
  }
  auto slotOf = [&](int k) { return rows ? b.slot(k) : stage; };
  auto readyOf = [&](int k) { return rows ? b.slotReady(k) : b.stagingReady(); };
  auto freeOf = [&](int k) { return rows ? b.slotFree(k) : b.stagingFree(); };
  st.route = rows ? "dma_ring" : "staged";
  st.buffers = static_cast<size_t>(slots);
  st.chunkBytes = static_cast<size_t>(rowsPer * rowBytes);
  // One status word for all chunks: cleared once here, read once at the end.
  if (l.needsStatus && !b.keepStatus) {
    const int rc = sbc_fill(b.statusWord(), 1, 4, 0, b.computeStream());
    if (rc) {
      b.fail("status reset", rc);
      return terr("backend_failure", b.error());
    }
  }
  struct Keep {
    CudaBackend &b;
    bool old;
    ~Keep() { b.keepStatus = old; }
  } keep{b, b.keepStatus};
  b.keepStatus = true;
  int64_t i = 0;
  for (int64_t r0 = 0; r0 < nrows; r0 += rowsPer, ++i) {
    const int64_t r1 = std::min(r0 + rowsPer, nrows);
    const int s = static_cast<int>(i % slots);
    void *slot = slotOf(s);
    int rc;
    if ((rc = sbc_stream_wait_event(b.computeStream(), freeOf(s)))) {
      b.fail("ring wait", rc);
      return terr("backend_failure", b.error());
    }
    if (auto e = runDevice(l, b, dsrc, slot, rows ? RowWindow{r0, r1} : RowWindow{}, st))
      return e;
    const size_t bytes = static_cast<size_t>((r1 - r0) * rowBytes);
    if ((rc = sbc_event_record(readyOf(s), b.computeStream())) ||
        (rc = sbc_stream_wait_event(b.copyStream(), readyOf(s))) ||
        (rc = sbc_memcpy_d2h_async(static_cast<uint8_t *>(hdst) + r0 * rowBytes, slot, bytes, b.copyStream())) ||
        (rc = sbc_event_record(freeOf(s), b.copyStream()))) {
      b.fail("ring download", rc);
      return terr("backend_failure", b.error());
    }
    ++b.copyCalls;
    ++st.copies;
    b.eventRecords += 2;
    b.eventWaits += 2;
    st.payloadBytes += static_cast<int64_t>(bytes);
    ++st.chunks;
  }
  return std::nullopt;
}

std::optional<TransferError> runSourceRows(const Lowered &l, CudaBackend &b, const void *rows, int64_t rowBegin,
                                           int64_t rowEnd, void *ddst, RunStats &st) {
  if (!l.rowsChunkable || l.srcOuter < 0)
    return terr("invalid_options", "the plan's source has no row axis (rows are not contiguous blocks)");
  const int ax = l.srcOuter;
  const int64_t E = l.desc.extents[ax], lo = l.desc.pad_lo[ax];
  if (rowBegin < 0 || rowEnd > E || rowEnd <= rowBegin)
    return terr("invalid_options", "source rows [" + std::to_string(rowBegin) + ", " + std::to_string(rowEnd) +
                                       ") outside [0, " + std::to_string(E) + ")");
  if (l.desc.has_fill && !l.denseCover)
    return terr("invalid_options", "source-row windows need a destination the result box covers densely");
  sbc_relocate d = l.desc;
  // the first / last window also produces the pad rows before / after it
  d.box_lo[ax] = rowBegin == 0 ? 0 : lo + rowBegin;
  d.box_hi[ax] = rowEnd == E ? l.padded[ax] : lo + rowEnd;
  if (auto e = uploadParams(l, b, d))
    return e;
  if (auto e = zeroStatus(l, b, d))
    return e;
  d.src = rows;
  d.src_offset = rowBegin * l.desc.src_strides[ax];
  d.dst = ddst;
  st.kernel = familyName(l.family);
  st.route = "device";
  return launch(l, b, d, st);
}

std::optional<TransferError> runSourceShards(const Lowered &l, CudaBackend &b, const void *const *shards,
                                             const int64_t *bounds, int n, void *ddst, RunStats &st) {
  if (!l.rowsChunkable || l.srcOuter < 0)
    return terr("invalid_options", "the plan's source has no row axis (rows are not contiguous blocks)");
  if (n < 1)
    return terr("invalid_options", "no source shards");
  const int64_t E = l.desc.extents[l.srcOuter];
  if (bounds[0] != 0 || bounds[n] != E)
    return terr("invalid_options", "source shards must cover rows [0, " + std::to_string(E) + ")");
  for (int j = 0; j < n; ++j)
    if (bounds[j + 1] < bounds[j])
      return terr("invalid_options", "source shard bounds must not decrease");
  // One tile launch over all shards when the plan is a rank-2 transpose whose
  // source rows are axis 1 and the shards fit the TMA tiles.
  if (l.family == Family::Transpose && l.desc.rank == 2 && l.srcOuter == 1 && n <= 8) {
    std::vector<const void *> srcs;
    std::vector<int64_t> rb;
    for (int j = 0; j < n; ++j)
      if (bounds[j + 1] > bounds[j]) {
        srcs.push_back(shards[j]);
        rb.push_back(bounds[j]);
      }
    rb.push_back(E);
    sbc_relocate d = l.desc;
    if (auto e = uploadParams(l, b, d))
      return e;
    if (auto e = zeroStatus(l, b, d))
      return e;
    d.dst = ddst;
    d.fault = b.faultWord();
    const int rc = sbc_relocate_transpose_shards(&d, srcs.data(), rb.data(), static_cast<int32_t>(srcs.size()),
                                                 b.computeStream());
    if (rc == 0) {
      ++st.launches;
      ++b.kernelLaunches;
      st.kernel = familyName(l.family);
      st.route = "device";
      return std::nullopt;
    }
    if (rc != SBC_EUNSUPPORTED) {
      b.fail("tile kernel over shards", rc);
      return terr("backend_failure", b.error());
    }
  }
  for (int j = 0; j < n; ++j)
    if (bounds[j + 1] > bounds[j])
      if (auto e = runSourceRows(l, b, shards[j], bounds[j], bounds[j + 1], ddst, st))
        return e;
  return std::nullopt;
}

Route chooseRoute(const Lowered &l, CudaBackend &b, const void *hsrc, const TransferOptions &o) {
  if (o.route != Route::Auto)
    return o.route;
  int kind = 0, dev = -1;
  void *mapped = nullptr;
  const bool pinned = sbc_pointer_info(hsrc, &kind, &dev) == 0 && kind == 1 &&
                      sbc_host_device_pointer(const_cast<void *>(hsrc), &mapped) == 0;
  if (!l.rowsChunkable)
    return pinned ? Route::ZeroCopy : Route::Staged;
  if (!pinned)
    return Route::DmaRing;
  auto &s = b.routeStats[l.classKey];
  // Zero copy is sampled first, so the cold samples of a fresh process (a
  // link leaving its idle state, first touch of the pinned source) fall on
  // it, and it must beat the copy-engine ring by 10 % to be chosen: in steady
  // state the ring measured faster on every plan class tried here.
  if (s.zeroCopySamples < 2)
    return Route::ZeroCopy;
  if (s.dmaSamples < 2)
    return Route::DmaRing;
  const bool zeroCopyFaster = s.zeroCopySecondsPerByte < 0.9 * s.dmaSecondsPerByte;
  return zeroCopyFaster != s.probe ? Route::ZeroCopy : Route::DmaRing;
}

std::optional<TransferError> runH2D(const Lowered &l, CudaBackend &b, const void *hsrc, void *ddst, Route route,
                                    RowWindow w, const TransferOptions &o, RunStats &st) {
  const int r = l.desc.rank;
  const int ws = l.desc.src_width;
  if (route == Route::ZeroCopy) {
    void *mapped = nullptr;
    const int rc = sbc_host_device_pointer(const_cast<void *>(hsrc), &mapped);
    if (rc)
      return terr("invalid_view", "zero_copy needs a mapped pinned host source");
    st.route = "zero_copy";
    st.payloadBytes += l.srcElements * ws; // upper bound: the window may read less
    return runDevice(l, b, mapped, ddst, w, st);
  }

  sbc_relocate base = l.desc;
  if (!applyWindow(l, base, w))
    return terr("invalid_options", "row window outside the padded result");
  if (auto e = uploadParams(l, b, base))
    return e;
  if (auto e = zeroStatus(l, b, base))
    return e;
  if (auto e = prefill(l, b, ddst, w, st))
    return e;
  base.dst = ddst;
  st.kernel = familyName(l.family);
  // Pageable (unregistered) sources of 1 MiB or more go through the
  // context's pinned bounce buffers (threaded host copy + DMA).
  int kind = -1, owner = -1;
  const bool bounce = static_cast<size_t>(l.srcElements) * ws >= (size_t(1) << 20) &&
                      sbc_pointer_info(hsrc, &kind, &owner) == 0 && kind == 0;
  auto upload = [&](void *dstDev, const void *srcHost, size_t bytes) -> int {
    if (!bounce)
      return sbc_memcpy_h2d_async(dstDev, srcHost, bytes, b.copyStream());
    if (!b.bounceH2D(dstDev, srcHost, bytes))
      return -1;
    --b.copyCalls; // counted once below, like a direct copy
    return 0;
  };

  // Chunk axis and source compaction mode.
  //  rows   : chunk = whole source rows along srcOuter (window on axis 0
  //           allowed only when srcOuter == 0): one contiguous DMA
  //  rows2d : rank-2 layout, window on axis 0 (source stride 1) and chunks
  //           along axis 1: one 2-D DMA of the window's columns per chunk
  //  whole  : one DMA of the entire source, one kernel
  enum class Mode { Rows, Rows2D, Whole } mode = Mode::Whole;
  const int o_ax = l.srcOuter;
  if (route != Route::Staged && l.rowsChunkable && o_ax >= 0) {
    if (isWhole(l, w) || o_ax == 0)
      mode = Mode::Rows;
    else if (r == 2 && o_ax == 1 && l.desc.src_strides[0] == 1)
      mode = Mode::Rows2D;
  }
  if (route == Route::Staged && r == 2 && o_ax == 1 && l.rowsChunkable && !isWhole(l, w) &&
      l.desc.src_strides[0] == 1)
    mode = Mode::Rows2D; // one chunk of the window's columns

  if (mode == Mode::Whole) {
    const size_t bytes = static_cast<size_t>(l.srcElements) * ws;
    auto sg = budgetedStaging(b, bytes);
    if (auto *e = std::get_if<TransferError>(&sg))
      return *e;
    void *stage = std::get<void *>(sg);
    int rc;
    if ((rc = sbc_stream_wait_event(b.copyStream(), b.stagingFree())) || (rc = upload(stage, hsrc, bytes)) ||
        (rc = sbc_event_record(b.stagingReady(), b.copyStream())) ||
        (rc = sbc_stream_wait_event(b.computeStream(), b.stagingReady()))) {
      b.fail("staged upload", rc);
      return terr("backend_failure", b.error());
    }
    ++b.copyCalls;
    ++st.copies;
    st.route = "staged";
    st.chunks = 1;
    st.chunkBytes = bytes;
    st.buffers = 1;
    st.payloadBytes += static_cast<int64_t>(bytes);
    sbc_relocate d = base;
    d.src = stage;
    if (auto e = launch(l, b, d, st))
      return e;
    if ((rc = sbc_event_record(b.stagingFree(), b.computeStream()))) {
      b.fail("staging release", rc);
      return terr("backend_failure", b.error());
    }
    return std::nullopt;
  }

  // Chunked ring.
  const int ax = mode == Mode::Rows ? o_ax : 1;
  const int64_t lo = l.desc.pad_lo[ax], E = l.desc.extents[ax];
  const int64_t B0 = base.box_lo[ax], B1 = base.box_hi[ax];
  const int64_t V0 = std::max(B0, lo), V1 = std::min(B1, lo + E); // valid padded rows in the box
  // Window columns (rows2d): valid source coordinates of axis 0.
  int64_t c0 = 0, c1 = 0;
  if (mode == Mode::Rows2D) {
    c0 = std::max<int64_t>(base.box_lo[0] - l.desc.pad_lo[0], 0);
    c1 = std::min<int64_t>(base.box_hi[0] - l.desc.pad_lo[0], l.desc.extents[0]);
    if (c1 < c0)
      c1 = c0;
  }
  const int64_t rowElems = mode == Mode::Rows ? l.desc.src_strides[ax] : (c1 - c0);
  const int64_t rowBytes = std::max<int64_t>(rowElems * ws, 1);
  // Default chunk: a quarter of the upload, 8 to 64 MiB. Every chunk costs a
  // copy-engine round (measured: 64 MiB f32 -> f16 takes 1.336 ms in 8 MiB
  // chunks, 1.318 ms in 32 MiB ones), and the kernels are fast enough that
  // the pipeline's tail (the last chunk's kernel) stays short.
  const size_t validBytes = static_cast<size_t>(std::max<int64_t>(V1 - V0, 0)) * static_cast<size_t>(rowBytes);
  size_t target = o.chunkSizeOverride ? o.chunkSizeOverride
                                      : std::clamp(validBytes / 4, kDefaultChunkBytes, kMaxChunkBytes);
  // Staged: the valid rows in one piece, in the staging buffer.
  const bool single = route == Route::Staged;
  const int slots = single ? 1 : std::max(2, o.nBuffers);
  void *stage = nullptr;
  int64_t rowsPer;
  if (single) {
    rowsPer = std::max<int64_t>(1, V1 - V0);
    auto sg = budgetedStaging(b, static_cast<size_t>(rowsPer * rowBytes));
    if (auto *e = std::get_if<TransferError>(&sg))
      return *e;
    stage = std::get<void *>(sg);
  } else {
    auto t = budgetedChunk(b, slots, target, rowBytes, !o.chunkSizeOverride);
    if (auto *e = std::get_if<TransferError>(&t))
      return *e;
    target = std::get<size_t>(t);
    rowsPer = std::max<int64_t>(1, static_cast<int64_t>(target) / rowBytes);
    // Chunk boundaries on a multiple of 128 (else 64) rows keep every
    // chunk's destination box 16-byte aligned and made of whole kernel tiles
    // (128 rows: the tall int8 tiles).
    rowsPer = wholeTileRows(rowsPer);
    if (!b.ensureRing(slots, static_cast<size_t>(rowsPer * rowBytes)))
      return terr("backend_failure", b.error());
  }
  st.route = route == Route::Staged ? "staged" : "dma_ring";
  st.buffers = static_cast<size_t>(slots);
  st.chunkBytes = static_cast<size_t>(rowsPer * rowBytes);

  if (V1 <= V0) { // the box holds only pad rows: no source needed
    sbc_relocate d = base;
    d.src = nullptr;
    st.chunks = 1;
    return launch(l, b, d, st);
  }
  int64_t i = 0;
  for (int64_t r0 = V0; r0 < V1; r0 += rowsPer, ++i) {
    const int64_t r1 = std::min(r0 + rowsPer, V1);
    const int s = static_cast<int>(i % slots);
    void *slot = single ? stage : b.slot(s);
    void *slotFree = single ? b.stagingFree() : b.slotFree(s);
    void *slotReady = single ? b.stagingReady() : b.slotReady(s);
    int rc;
    if ((rc = sbc_stream_wait_event(b.copyStream(), slotFree))) {
      b.fail("ring wait", rc);
      return terr("backend_failure", b.error());
    }
    const int64_t v0 = r0 - lo, v1 = r1 - lo; // source rows
    if (mode == Mode::Rows) {
      const auto *src = static_cast<const uint8_t *>(hsrc) + v0 * rowBytes;
      rc = upload(slot, src, static_cast<size_t>((v1 - v0) * rowBytes));
    } else {
      const int64_t S1 = l.desc.src_strides[1];
      const auto *src = static_cast<const uint8_t *>(hsrc) + (v0 * S1 + c0) * ws;
      rc = sbc_memcpy_h2d_2d_async(slot, static_cast<size_t>(rowBytes), src, static_cast<size_t>(S1 * ws),
                                   static_cast<size_t>((c1 - c0) * ws), static_cast<size_t>(v1 - v0), b.copyStream());
    }
    if (rc || (rc = sbc_event_record(slotReady, b.copyStream())) ||
        (rc = sbc_stream_wait_event(b.computeStream(), slotReady))) {
      b.fail("ring upload", rc);
      return terr("backend_failure", b.error());
    }
    ++b.copyCalls;
    ++st.copies;
    b.eventRecords += 1;
    b.eventWaits += 2;
    st.payloadBytes += (v1 - v0) * rowBytes;
    sbc_relocate d = base;
    d.box_lo[ax] = (r0 == V0) ? B0 : r0;
    d.box_hi[ax] = (r1 == V1) ? B1 : r1;
    d.src = slot;
    if (mode == Mode::Rows) {
      d.src_offset = v0 * l.desc.src_strides[ax];
    } else {
      d.src_strides[1] = c1 - c0;
      d.src_offset = v0 * (c1 - c0) + c0;
    }
    if (auto e = launch(l, b, d, st))
      return e;
    if ((rc = sbc_event_record(slotFree, b.computeStream()))) {
      b.fail("ring release", rc);
      return terr("backend_failure", b.error());
    }
    ++b.eventRecords;
  }
  st.chunks = static_cast<size_t>(i);
  return std::nullopt;
}

std::optional<TransferError> runH2DStatic(const Lowered &l, const void *hsrc, void *ddst, void *stream,
                                          uint8_t *scratch, size_t scratchBytes) {
  // Scratch layout: [0, 4) status word, [4, 8) fault word (in [0, 256)) |
  // [256, 256 + kParams) parameters | the rest one staging slot for source rows.
  constexpr size_t kStatus = 256, kParams = size_t(1) << 20;
  if (l.paramBlob.size() > kParams)
    return terr("invalid_options", "parameters exceed the static scratch's 1 MiB parameter area (" +
                                       std::to_string(l.paramBlob.size()) + " bytes)");
  uint8_t *slot = scratch + kStatus + kParams;
  const size_t slotBytes = scratchBytes - kStatus - kParams;
  sbc_relocate base = l.desc;
  int rc = 0;
  if (!l.paramBlob.empty()) {
    uint8_t *pdev = scratch + kStatus;
    if ((rc = sbc_memcpy_h2d_async(pdev, l.paramBlob.data(), l.paramBlob.size(), stream)))
      return terr("backend_failure", std::string("parameter copy: ") + sbc_error_string(rc));
    for (int k = 0; k < base.nstages; ++k) {
      if (l.paramOffset[static_cast<size_t>(k)] != kNone)
        base.stages[k].param = reinterpret_cast<const float *>(pdev + l.paramOffset[static_cast<size_t>(k)]);
      if (l.zpOffset[static_cast<size_t>(k)] != kNone)
        base.stages[k].zero_point = reinterpret_cast<const int32_t *>(pdev + l.zpOffset[static_cast<size_t>(k)]);
    }
  }
  // The scratch keeps the previous call's contents: the status and fault words
  // must start at 0 (one 8-byte fill covers both).
  if (l.needsStatus)
    base.status = reinterpret_cast<int32_t *>(scratch);
  base.fault = reinterpret_cast<int32_t *>(scratch + 4);
  if ((rc = sbc_fill(scratch, 2, 4, 0, stream)))
    return terr("backend_failure", std::string("status reset: ") + sbc_error_string(rc));
  const uint64_t waits0 = sbc_wait_launch_count();
  if (l.desc.has_fill && !l.denseCover &&
      (rc = sbc_fill(ddst, l.dstElements, l.desc.dst_width, l.desc.fill_bits, stream)))
    return terr("backend_failure", std::string("fill kernel: ") + sbc_error_string(rc));
  base.dst = ddst;
  const int ws = l.desc.src_width;
  auto launchOn = [&](const sbc_relocate &d) -> int { return launchFamily(l.family, d, stream); };
  if (!l.rowsChunkable || l.srcOuter < 0) {
    const size_t bytes = static_cast<size_t>(l.srcElements) * ws;
    if (bytes > slotBytes)
      return terr("invalid_options", "source of " + std::to_string(bytes) +
                                         " bytes is not row-chunkable and exceeds the static scratch's " +
                                         std::to_string(slotBytes) + "-byte staging slot");
    if ((rc = sbc_memcpy_h2d_async(slot, hsrc, bytes, stream)))
      return terr("backend_failure", std::string("source copy: ") + sbc_error_string(rc));
    sbc_relocate d = base;
    d.src = slot;
    if ((rc = launchOn(d)))
      return terr("backend_failure", std::string("relocation kernel: ") + sbc_error_string(rc));
  } else {
    const int ax = l.srcOuter;
    const int64_t lo = l.desc.pad_lo[ax], E = l.desc.extents[ax];
    const int64_t B1 = l.padded[ax];
    const int64_t rowBytes = l.desc.src_strides[ax] * ws;
    int64_t rowsPer = static_cast<int64_t>(slotBytes) / rowBytes;
    if (rowsPer < 1)
      return terr("invalid_options", "one source row of " + std::to_string(rowBytes) +
                                         " bytes exceeds the static scratch's " + std::to_string(slotBytes) +
                                         "-byte staging slot");
    rowsPer = wholeTileRows(rowsPer);
    for (int64_t r0 = lo; r0 < lo + E; r0 += rowsPer) {
      const int64_t r1 = std::min(r0 + rowsPer, lo + E);
      const int64_t v0 = r0 - lo, v1 = r1 - lo;
      // Same stream: this copy starts only after the previous chunk's kernel.
      if ((rc = sbc_memcpy_h2d_async(slot, static_cast<const uint8_t *>(hsrc) + v0 * rowBytes,
                                     static_cast<size_t>((v1 - v0) * rowBytes), stream)))
        return terr("backend_failure", std::string("source copy: ") + sbc_error_string(rc));
      sbc_relocate d = base;
      d.box_lo[ax] = r0 == lo ? 0 : r0;
      d.box_hi[ax] = r1 == lo + E ? B1 : r1;
      d.src = slot;
      d.src_offset = v0 * l.desc.src_strides[ax];
      if ((rc = launchOn(d)))
        return terr("backend_failure", std::string("relocation kernel: ") + sbc_error_string(rc));
    }
  }
  // A kernel with bounded waits ran (this call's, or another thread's at the
  // same time: then the read is only unneeded): wait for the stream and read
  // the fault word with the status word.
  const bool waited = sbc_wait_launch_count() != waits0;
  if (l.needsStatus || waited) {
    int32_t words[2] = {0, 0};
    if ((rc = sbc_memcpy_d2h_async(words, scratch, sizeof(words), stream)) || (rc = sbc_stream_synchronize(stream)))
      return terr("backend_failure", std::string("status readback: ") + sbc_error_string(rc));
    if (words[1])
      return terr("backend_failure", "a kernel's bounded wait for a TMA copy ran out; the output is incomplete");
    if (words[0])
      return terr("channel_out_of_range", "a channel index fell outside its parameter table");
  }
  return std::nullopt;
}

} // namespace b200
} // namespace reloc
