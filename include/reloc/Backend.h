// sym_b200 -- the copy-backend interface that execution entry points take
// (reference: libreloc/include/reloc/Backend.h:34-89). The names, signatures
// and contract are the reference's so that C++ callers written against it
// compile unchanged: no exceptions cross the interface, failures are sticky
// (failed() / error()), quiesce() establishes completion without relying on a
// recorded event, waitStream() orders every private queue after a caller's
// stream.
//
// Only reloc::CudaBackend (reloc/CudaBackend.h) executes plans here: the
// B200 executor runs no plan on the CPU, so executeDispatch and
// executeTransfer answer any other backend with `backend_mismatch` before
// doing any work.
#ifndef SYM_B200_RELOC_BACKEND_H
#define SYM_B200_RELOC_BACKEND_H

#include <cstddef>
#include <cstdint>
#include <string>

namespace reloc {

/// Direction of one asynchronous copy: for HostToDevice `dst` is device
/// memory and `src` host staging; DeviceToHost swaps them.
enum class CopyDir { HostToDevice, DeviceToHost };

/// Whether everything submitted to a backend's queues has finished. Unknown
/// never allows reusing or freeing memory that work touched.
enum class QueueCompletion { Complete, Unknown };

/// Opaque completion handle; 0 is "no event" (waits and queries return at
/// once). A failed recordEvent may return 0 after work was enqueued.
using EventHandle = uint64_t;

class CopyBackend {
public:
  virtual ~CopyBackend() = default;

  /// Host staging of `bytes` (pinned for CUDA); nullptr on failure.
  virtual void *allocStaging(size_t bytes) = 0;
  virtual void freeStaging(void *p) = 0;

  /// Logical queues (CUDA streams); at least 1.
  virtual int numQueues() const = 0;

  /// Enqueue an asynchronous copy on `queue`; copies of one queue complete in
  /// order.
  virtual void copyAsync(int queue, void *dst, const void *src, size_t bytes, CopyDir dir) = 0;

  /// An event after everything enqueued so far on `queue`.
  virtual EventHandle recordEvent(int queue) = 0;

  /// Block until `ev` completed, then retire it (0 and retired handles
  /// return at once). Check failed() too: a failed wait proves nothing.
  virtual void waitEvent(EventHandle ev) = 0;

  /// true once `ev` completed (or ev == 0); never blocks.
  virtual bool queryEvent(EventHandle ev) = 0;

  /// Drain every owned queue, even after earlier failures; Unknown when any
  /// queue cannot be proven complete. The first error() is kept apart from
  /// this result. Callers stop submitting before calling it.
  virtual QueueCompletion quiesce() = 0;

  /// Order every private queue after the work already on an external stream
  /// (a caller's cudaStream_t, erased to void*). false (with the error
  /// recorded) on failure; backends without streams return true.
  virtual bool waitStream(const void * /*externalStream*/) { return true; }

  /// Sticky: true once any operation of this backend failed.
  virtual bool failed() const { return false; }

  /// The first recorded failure; empty while there is none.
  virtual const std::string &error() const {
    static const std::string none;
    return none;
  }

  /// The CUDA device of this backend's queues; -1 for host-only backends.
  virtual int device() const { return -1; }
};

} // namespace reloc

#endif
