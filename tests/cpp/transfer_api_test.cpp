// A C++ caller of the runtime API (include/reloc/*.h), compiled against the
// headers and linked to libsb_runtime.so with no C-ABI in between: the
// boundary a C++ program written against the reference's libreloc headers
// uses (Decode.h, Bind.h, Transfer.h, Dispatch.h, Backend.h).
//
//   transfer_api_test cpu <c1.blob> <c4.blob>
//       validation and backend checks that need no GPU; prints one line per
//       check and "cpu ok" at the end (exit 0), or the failing check (exit 1).
//   transfer_api_test gpu <c1.blob> <N> <c1_src> <c1_h2d_out> <c1_d2h_out>
//                         <c4.blob> <out> <in> <c4_src> <c4_scale> <c4_out>
//       config 1 (layout plan, symbol N) through executeTransfer host-to-device
//       and device-to-host, and config 4's plan (int8 [out, in] + per-row
//       scale -> f16 [in, out]) through executeDispatch with the backend
//       passed as a CopyBackend&; writes the result bytes for the caller to
//       compare with the reference executor.
#include "reloc/Backend.h"
#include "reloc/Bind.h"
#include "reloc/CudaBackend.h"
#include "reloc/Decode.h"
#include "reloc/Dispatch.h"
#include "reloc/Transfer.h"

#include "sb_cuda.h"

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <iterator>
#include <string>
#include <vector>

using namespace reloc;

namespace {

std::vector<uint8_t> readFile(const char *path) {
  std::ifstream f(path, std::ios::binary);
  return std::vector<uint8_t>(std::istreambuf_iterator<char>(f), {});
}

bool writeFile(const char *path, const void *data, size_t n) {
  std::FILE *f = std::fopen(path, "wb");
  if (!f)
    return false;
  const bool ok = std::fwrite(data, 1, n, f) == n;
  std::fclose(f);
  return ok;
}

int failures = 0;

void expect(bool ok, const std::string &what) {
  std::printf("%s %s\n", ok ? "pass" : "FAIL", what.c_str());
  if (!ok)
    ++failures;
}

template <class V> std::string codeOf(const V &v) {
  if (auto *e = std::get_if<TransferError>(&v))
    return e->code;
  return "ok";
}

std::string codeOf(const std::optional<TransferError> &e) { return e ? e->code : std::string("ok"); }

/// A host-only backend: every B200 entry point must refuse it.
class HostOnlyBackend : public CopyBackend {
public:
  void *allocStaging(size_t bytes) override { return std::malloc(bytes); }
  void freeStaging(void *p) override { std::free(p); }
  int numQueues() const override { return 1; }
  void copyAsync(int, void *dst, const void *src, size_t bytes, CopyDir) override { std::memcpy(dst, src, bytes); }
  EventHandle recordEvent(int) override { return 0; }
  void waitEvent(EventHandle) override {}
  bool queryEvent(EventHandle) override { return true; }
  QueueCompletion quiesce() override { return QueueCompletion::Complete; }
};

BoundPlan bindC1(const std::vector<uint8_t> &blob, int64_t n) {
  auto plan = decodePlan(blob.data(), blob.size());
  if (auto *e = std::get_if<DecodeError>(&plan)) {
    std::printf("FAIL decode: %s\n", e->message.c_str());
    std::exit(1);
  }
  auto bound = bind(std::get<RelocationPlan>(plan), SymbolMap{{"N", n}});
  if (auto *e = std::get_if<BindError>(&bound)) {
    std::printf("FAIL bind: %s\n", e->message.c_str());
    std::exit(1);
  }
  return std::get<BoundPlan>(bound);
}

BufferView view(const void *base, size_t capacity, std::vector<int64_t> extents, std::vector<int64_t> strides,
                uint32_t width, MemoryKind kind, int device) {
  BufferView v;
  v.base = reinterpret_cast<uintptr_t>(base);
  v.capacityBytes = capacity;
  v.extents = std::move(extents);
  v.strides = std::move(strides);
  v.elementSize = width;
  v.kind = kind;
  v.device = device;
  return v;
}

int cpuChecks(const char *c1Path, const char *c4Path) {
  const auto c1 = readFile(c1Path);
  const int64_t n = 4096;
  const BoundPlan b = bindC1(c1, n);
  std::vector<float> host(n), other(n);
  uint8_t fakeDevice[16]; // never dereferenced: validation only reads the declaration
  const BufferView src = view(host.data(), n * 4, {n}, {1}, 4, MemoryKind::Host, -1);
  const BufferView dst = view(fakeDevice, n * 4, {64, n / 64}, {n / 64, 1}, 4, MemoryKind::Cuda, 0);

  auto ok = validateTransfer(b, src, dst, TransferDirection::HostToDevice);
  expect(codeOf(ok) == "ok", "validateTransfer accepts the plan's dense views");
  if (auto *r = std::get_if<TransferRequest>(&ok)) {
    expect(r->sourceSpanBytes == static_cast<size_t>(n * 4), "source span is the whole source");
    expect(r->destinationBytes == static_cast<size_t>(n * 4), "destination bytes are the plan's");
  }
  BufferView v = src;
  v.base = 0;
  expect(codeOf(validateTransfer(b, v, dst, TransferDirection::HostToDevice)) == "invalid_view", "null base");
  v = src;
  v.extents = {2, n / 2};
  v.strides = {1, 1};
  expect(codeOf(viewSpanBytes(v, "source")) == "unsupported_layout", "overlapping strides");
  v.strides = {0, 1};
  expect(codeOf(viewSpanBytes(v, "source")) == "unsupported_layout", "broadcast stride");
  v.strides = {-1, 2};
  expect(codeOf(viewSpanBytes(v, "source")) == "unsupported_layout", "negative stride");
  v = src;
  v.capacityBytes = n * 4 - 1;
  expect(codeOf(validateTransfer(b, v, dst, TransferDirection::HostToDevice)) == "insufficient_capacity",
         "source capacity below its span");
  v = src;
  v.extents = {n - 1};
  expect(codeOf(validateTransfer(b, v, dst, TransferDirection::HostToDevice)) == "plan_mismatch",
         "source holds fewer elements than the plan moves");
  v = src;
  v.kind = MemoryKind::Cuda;
  v.device = 0;
  expect(codeOf(validateTransfer(b, v, dst, TransferDirection::HostToDevice)) == "direction_mismatch",
         "host-to-device source in CUDA memory");
  BufferView d = dst;
  d.strides = {1, 64};
  expect(codeOf(validateTransfer(b, src, d, TransferDirection::HostToDevice)) == "unsupported_layout",
         "destination not dense");
  d = dst;
  d.extents = {64, n / 64 - 1};
  d.strides = {n / 64 - 1, 1};
  expect(codeOf(validateTransfer(b, src, d, TransferDirection::HostToDevice)) == "plan_mismatch",
         "destination smaller than the plan writes");

  // typed plans' layouts are refused by the layout path
  const auto c4 = readFile(c4Path);
  auto tplan = decodeTypedPlan(c4.data(), c4.size());
  expect(std::holds_alternative<TypedRelocationPlan>(tplan), "decodeTypedPlan accepts config 4's plan");
  ParameterMap params;
  ParameterValue scale;
  scale.elementType = ElementType{ElementTypeKind::Float, 32};
  scale.extents = {64};
  const float one = 1.0f;
  for (int i = 0; i < 64; ++i)
    scale.bytes.insert(scale.bytes.end(), reinterpret_cast<const uint8_t *>(&one),
                       reinterpret_cast<const uint8_t *>(&one) + 4);
  params["scale"] = scale;
  auto tb = bindTyped(std::get<TypedRelocationPlan>(tplan), SymbolMap{{"out_features", 64}, {"in_features", 128}},
                      params);
  if (auto *be = std::get_if<BindError>(&tb)) {
    expect(false, "bindTyped binds config 4's plan: " + be->message);
    return 1;
  }
  const TypedBoundPlan &typed = std::get<TypedBoundPlan>(tb);
  std::vector<int8_t> q(64 * 128);
  const BufferView qsrc = view(q.data(), q.size(), {64 * 128}, {1}, 1, MemoryKind::Host, -1);
  const BufferView qdst = view(fakeDevice, 64 * 128 * 1, {64 * 128}, {1}, 1, MemoryKind::Cuda, 0);
  expect(codeOf(validateTransfer(typed.layout, qsrc, qdst, TransferDirection::HostToDevice)) == "typed_unsupported",
         "the layout of a typed plan is refused");

  // every execution entry point refuses a host-only backend, before any work
  HostOnlyBackend host_only;
  auto req = validateTransfer(b, src, dst, TransferDirection::HostToDevice);
  auto &tr = std::get<TransferRequest>(req);
  expect(codeOf(executeTransfer(tr, host_only, TransferOptions{})) == "backend_mismatch",
         "executeTransfer on a host-only backend");
  expect(!tr.consumed, "a refused transfer request stays unconsumed");
  dispatch::Options o;
  o.cuda = true;
  auto tmpl = dispatch::prepareDispatchTemplate(typed, TransferDirection::HostToDevice, o);
  expect(std::holds_alternative<dispatch::DispatchTemplate>(tmpl), "prepareDispatchTemplate selects a B200 row");
  const BufferView tsrc = view(q.data(), q.size(), {64, 128}, {128, 1}, 1, MemoryKind::Host, -1);
  const BufferView tdst = view(fakeDevice, 64 * 128 * 2, {128, 64}, {64, 1}, 2, MemoryKind::Cuda, 0);
  auto dreq = dispatch::prepareDispatch(std::get<dispatch::DispatchTemplate>(tmpl), tsrc, tdst);
  expect(std::holds_alternative<dispatch::DispatchRequest>(dreq), "prepareDispatch validates the views");
  auto &dr = std::get<dispatch::DispatchRequest>(dreq);
  CopyBackend &generic = host_only;
  expect(codeOf(dispatch::executeDispatch(dr, generic, TransferOptions{})) == "backend_mismatch",
         "executeDispatch(CopyBackend&) on a host-only backend");
  expect(!dr.consumed, "a refused dispatch request stays unconsumed");
  tr.consumed = true;
  expect(codeOf(executeTransfer(tr, host_only, TransferOptions{})) == "already_executed",
         "a consumed transfer request");
  std::printf(failures ? "cpu FAILED\n" : "cpu ok\n");
  return failures ? 1 : 0;
}

int gpuRun(char **a) {
  const auto c1 = readFile(a[0]);
  const int64_t n = std::atoll(a[1]);
  const auto c1src = readFile(a[2]);
  std::string err;
  auto backend = CudaBackend::create(0, err);
  if (!backend) {
    std::printf("FAIL CudaBackend::create: %s\n", err.c_str());
    return 1;
  }
  CopyBackend &generic = *backend;
  const size_t bytes = static_cast<size_t>(n) * 4;
  void *hostIn = nullptr, *hostOut = nullptr, *dev = nullptr, *dev2 = nullptr;
  if (sbc_malloc_host(&hostIn, bytes, 0) || sbc_malloc_host(&hostOut, bytes, 0) || sbc_malloc_device(&dev, bytes) ||
      sbc_malloc_device(&dev2, bytes)) {
    std::printf("FAIL allocation\n");
    return 1;
  }
  std::memcpy(hostIn, c1src.data(), bytes);
  const BoundPlan b = bindC1(c1, n);
  // host -> device
  auto req = validateTransfer(b, view(hostIn, bytes, {n}, {1}, 4, MemoryKind::Host, -1),
                              view(dev, bytes, {64, n / 64}, {n / 64, 1}, 4, MemoryKind::Cuda, 0),
                              TransferDirection::HostToDevice);
  expect(codeOf(req) == "ok", "validateTransfer host-to-device");
  auto e = executeTransfer(std::get<TransferRequest>(req), generic, TransferOptions{});
  expect(!e, "executeTransfer host-to-device" + (e ? ": " + e->code + " " + e->message : std::string()));
  expect(codeOf(executeTransfer(std::get<TransferRequest>(req), generic, TransferOptions{})) == "already_executed",
         "requests are single-use");
  std::vector<uint8_t> out(bytes);
  sbc_memcpy_d2h_async(out.data(), dev, bytes, nullptr);
  sbc_stream_synchronize(nullptr);
  writeFile(a[3], out.data(), bytes);
  // device -> host: the source (the original values) on the device
  sbc_memcpy_h2d_async(dev2, c1src.data(), bytes, nullptr);
  sbc_stream_synchronize(nullptr);
  std::memset(hostOut, 0, bytes);
  auto back = validateTransfer(b, view(dev2, bytes, {n}, {1}, 4, MemoryKind::Cuda, 0),
                               view(hostOut, bytes, {64, n / 64}, {n / 64, 1}, 4, MemoryKind::Host, -1),
                               TransferDirection::DeviceToHost);
  expect(codeOf(back) == "ok", "validateTransfer device-to-host");
  e = executeTransfer(std::get<TransferRequest>(back), generic, TransferOptions{});
  expect(!e, "executeTransfer device-to-host" + (e ? ": " + e->code + " " + e->message : std::string()));
  writeFile(a[4], hostOut, bytes);

  // config 4's typed plan through executeDispatch(..., CopyBackend&, ...)
  const auto c4 = readFile(a[5]);
  const int64_t outF = std::atoll(a[6]), inF = std::atoll(a[7]);
  const auto q = readFile(a[8]);
  const auto s = readFile(a[9]);
  auto tplan = decodeTypedPlan(c4.data(), c4.size());
  ParameterMap params;
  ParameterValue scale;
  scale.elementType = ElementType{ElementTypeKind::Float, 32};
  scale.extents = {outF};
  scale.bytes = s;
  params["scale"] = scale;
  auto tb = bindTyped(std::get<TypedRelocationPlan>(tplan), SymbolMap{{"out_features", outF}, {"in_features", inF}},
                      params);
  dispatch::Options o;
  o.cuda = true;
  auto tmpl = dispatch::prepareDispatchTemplate(std::get<TypedBoundPlan>(tb), TransferDirection::HostToDevice, o);
  const size_t qBytes = q.size(), rBytes = static_cast<size_t>(outF * inF * 2);
  void *qHost = nullptr, *rDev = nullptr;
  if (sbc_malloc_host(&qHost, qBytes, 0) || sbc_malloc_device(&rDev, rBytes)) {
    std::printf("FAIL allocation\n");
    return 1;
  }
  std::memcpy(qHost, q.data(), qBytes);
  auto dreq = dispatch::prepareDispatch(std::get<dispatch::DispatchTemplate>(tmpl),
                                        view(qHost, qBytes, {outF, inF}, {inF, 1}, 1, MemoryKind::Host, -1),
                                        view(rDev, rBytes, {inF, outF}, {outF, 1}, 2, MemoryKind::Cuda, 0));
  expect(codeOf(dreq) == "ok", "prepareDispatch config 4");
  e = dispatch::executeDispatch(std::get<dispatch::DispatchRequest>(dreq), generic, TransferOptions{});
  expect(!e, "executeDispatch(CopyBackend&) config 4" + (e ? ": " + e->code + " " + e->message : std::string()));
  std::vector<uint8_t> r(rBytes);
  sbc_memcpy_d2h_async(r.data(), rDev, rBytes, nullptr);
  sbc_stream_synchronize(nullptr);
  writeFile(a[10], r.data(), rBytes);
  expect(!backend->failed(), "the backend is healthy afterwards");
  backend.reset();
  sbc_free_host(hostIn);
  sbc_free_host(hostOut);
  sbc_free_host(qHost);
  sbc_free_device(dev);
  sbc_free_device(dev2);
  sbc_free_device(rDev);
  std::printf(failures ? "gpu FAILED\n" : "gpu ok\n");
  return failures ? 1 : 0;
}

} // namespace

int main(int argc, char **argv) {
  if (argc == 4 && std::strcmp(argv[1], "cpu") == 0)
    return cpuChecks(argv[2], argv[3]);
  if (argc == 13 && std::strcmp(argv[1], "gpu") == 0)
    return gpuRun(argv + 2);
  std::fprintf(stderr, "usage: transfer_api_test cpu <c1.blob> <c4.blob> | gpu ...\n");
  return 2;
}
