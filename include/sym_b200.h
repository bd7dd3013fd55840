/* sym_b200 -- the drop-in C-ABI of the B200 typed relocation executor
 * (libsb_runtime.so).
 *
 * Plain pointers, sizes, POD structs and opaque handles; no CUDA, C++ or
 * torch type crosses it. Each entry point replaces one call of the
 * reference's Python binding `pyreloc` (libreloc/python/Py*.cpp), which is
 * what the reference's FFI binds for this path; the Python mirror in
 * sym_b200/pyreloc.py binds these through ctypes. Status: 0 = success,
 * otherwise non-zero with `err` filled (a stable code from the reference's
 * vocabulary, a message and, for decode errors, the byte offset).
 *
 * Ownership: handles are released with their *_free function. Parameter
 * bytes are copied at bind time. Buffers passed to the execute calls are
 * borrowed for the call (or, with async completion, until the caller's
 * stream passes the recorded completion).
 */
#ifndef SYM_B200_H
#define SYM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct sb_plan sb_plan;           /* a decoded wire v0 or v1 plan */
typedef struct sb_bound sb_bound;         /* a bound plan (typed: also its checked program) */
typedef struct sb_template sb_template;   /* a prepared dispatch template (no buffers) */
typedef struct sb_request sb_request;     /* a single-use prepared request */
typedef struct sb_resources sb_resources; /* typed contexts (per-device streams, HBM ring) */

typedef struct {
  char code[48];     /* e.g. "decode_error", "bind_error", "plan_mismatch" */
  char message[456];
  int64_t offset;    /* byte offset of a decode error, else -1 */
} sb_error;

/* A caller buffer (reference BufferView, libreloc/include/reloc/Transfer.h:47-56). */
typedef struct {
  uint64_t base;           /* allocation base address */
  uint64_t capacity_bytes;
  uint64_t offset_bytes;   /* logical element 0 */
  int32_t kind;            /* 0 host, 1 cuda */
  int32_t device;          /* CUDA ordinal, -1 for host */
  int32_t rank;            /* <= 8 */
  uint32_t element_size;
  int64_t extents[8];
  int64_t strides[8];      /* elements */
} sb_view;

/* Execution options (reference TransferOptions, Transfer.h:121-155, plus the route). */
typedef struct {
  int32_t n_buffers;          /* HBM ring slots; <= 0 = 4 */
  int32_t route;              /* 0 auto, 1 dma_ring, 2 zero_copy, 3 staged */
  uint64_t chunk_bytes;       /* ring slot bytes; 0 = heuristic */
  const void *caller_stream;  /* cudaStream_t of the caller, or NULL */
  int32_t has_caller_stream;  /* order after / signal caller_stream */
  int32_t async_completion;   /* return once enqueued; the caller stream carries completion */
} sb_options;

/* Version string of this library. */
const char *sb_version(void);
/* Kernels launched by this process through the library (instrumentation). */
uint64_t sb_kernel_launches(void);

/* pyreloc.wire_version (PyReloc.cpp:799): the blob's version or -1. */
int sb_wire_version(const uint8_t *data, size_t size);
/* pyreloc.load_plan (PyReloc.cpp:596): wire v0 -> decodePlan. */
int sb_load_plan(const uint8_t *data, size_t size, sb_plan **out, sb_error *err);
/* pyreloc.load_typed_plan (PyReloc.cpp:921): wire v1 -> decodeTypedPlan. */
int sb_load_typed_plan(const uint8_t *data, size_t size, sb_plan **out, sb_error *err);
/* TypedPlanHandle / PlanHandle properties as JSON (PyReloc.cpp:577-594, 812-862).
 * Returns the JSON length; writes at most cap-1 bytes plus NUL. */
int sb_plan_describe(const sb_plan *plan, char *json, size_t cap);
void sb_plan_free(sb_plan *plan);

/* pyreloc.bind (PyReloc.cpp:674): a v0 plan against {symbol: value}. */
int sb_bind(const sb_plan *plan, int32_t nsym, const char *const *names, const int64_t *values, sb_bound **out,
            sb_error *err);
/* pyreloc.bind_typed (PyReloc.cpp:987): a v1 plan against symbols and runtime
 * parameters (per parameter: name, dtype name, rank 0/1, extent, LE bytes). */
int sb_bind_typed(const sb_plan *plan, int32_t nsym, const char *const *names, const int64_t *values, int32_t nparam,
                  const char *const *pnames, const char *const *pdtypes, const int32_t *pranks,
                  const int64_t *pextents, const void *const *pbytes, const size_t *plens, sb_bound **out,
                  sb_error *err);
/* BoundPlan / TypedBoundPlan properties as JSON (layout, cuts, footprints,
 * stages with their checked arithmetic). */
int sb_bound_describe(const sb_bound *bound, char *json, size_t cap);
void sb_bound_free(sb_bound *bound);

/* pyreloc.query_capability (PyDispatch.cpp:831): JSON {eligible, excluded}.
 * direction: 0 h2d, 1 d2h. */
int sb_query_capability(const sb_bound *bound, int32_t direction, int32_t cuda, char *json, size_t cap,
                        sb_error *err);
/* pyreloc.prepare_dispatch_template (PyDispatch.cpp:612). policy: 0 auto,
 * 1 original_cpu; implementation: explicit row label or NULL/"". */
int sb_prepare_dispatch_template(const sb_bound *bound, int32_t direction, int32_t policy, const char *implementation,
                                 sb_template **out, sb_error *err);
/* pyreloc.make_transfer (PyTransfer.cpp:440) for wire v0 layout plans: a
 * template whose source is the dense 1-D span the plan reads and whose
 * result is the dense padded destination; executed like a typed template. */
int sb_prepare_transfer_template(const sb_bound *bound, sb_template **out, sb_error *err);
/* capability + selection as JSON. */
int sb_template_describe(const sb_template *tmpl, char *json, size_t cap);
void sb_template_free(sb_template *tmpl);

/* pyreloc.prepare_dispatch_from_template (PyDispatch.cpp:620): validate the
 * caller's views against the template. */
int sb_prepare_dispatch(const sb_template *tmpl, const sb_view *source, const sb_view *destination, sb_request **out,
                        sb_error *err);
/* pyreloc.execute_dispatch (PyDispatch.cpp:889): run the request on the
 * context of the destination's device (resources may be NULL: a private
 * context for this call). report: JSON of the reference Report fields. */
int sb_execute_dispatch(sb_request *request, sb_resources *resources, const sb_options *options, char *report,
                        size_t cap, sb_error *err);
void sb_request_free(sb_request *request);

/* Shard execution (reference typed::executeHostChunk contract,
 * TypedExecute.h:160-170, on the device): produce the physical rows
 * [row_begin, row_end) of axis 0 of the padded result into `dst` (the
 * window's own device storage, (row_end-row_begin) rows). host_source != 0:
 * `src` is the whole host source and only the rows' source bytes cross PCIe;
 * host_source == 0: `src` is the whole source in this device's memory. */
int sb_execute_rows(const sb_template *tmpl, sb_resources *resources, int32_t device, const void *src,
                    int32_t host_source, void *dst, int64_t row_begin, int64_t row_end, const sb_options *options,
                    char *report, size_t cap, sb_error *err);

/* The source-row counterpart of sb_execute_rows, for shards that are split
 * by source rows instead of result rows: `src` is device memory -- this
 * GPU's, or another GPU's mapped with sb_ipc_open -- holding source rows
 * [row_begin, row_end) of the plan's source-outer axis (dense, contiguous);
 * the kernel writes the result cells those rows produce into the full
 * destination `dst` on `device`. Disjoint windows, read from the GPUs that
 * hold them, assemble the whole result (the multi-GPU weight fetch reads
 * its peers' int8 shards over NVLink this way). */
int sb_execute_source_rows(const sb_template *tmpl, sb_resources *resources, int32_t device, const void *src,
                           int64_t row_begin, int64_t row_end, void *dst, const sb_options *options, char *report,
                           size_t cap, sb_error *err);

/* All of the source's rows as `n` consecutive blocks, block j at
 * `srcs[j]` holding rows [row_bounds[j], row_bounds[j+1]) (row_bounds[0] = 0,
 * row_bounds[n] = the source row count), each in device memory of this GPU or
 * of a peer (sb_ipc_open): the whole result is written to `dst` on `device`,
 * in ONE tile launch when the plan is a rank-2 transpose and the blocks fit
 * the TMA tiles, else one launch per block. */
int sb_execute_source_shards(const sb_template *tmpl, sb_resources *resources, int32_t device,
                             const void *const *srcs, const int64_t *row_bounds, int32_t n, void *dst,
                             const sb_options *options, char *report, size_t cap, sb_error *err);

/* CUDA IPC between the processes of a multi-GPU job (one per GPU): the
 * 64-byte handle of the device allocation holding `device_ptr` and the
 * pointer's byte offset in it; the allocation's mapping into this process on
 * `device` (returns its base: add the offset; peer access enabled); the
 * unmapping. */
int sb_ipc_handle(void *device_ptr, uint8_t handle[64], uint64_t *offset, sb_error *err);
int sb_ipc_open(const uint8_t handle[64], int32_t device, void **device_ptr, sb_error *err);
int sb_ipc_close(void *device_ptr, sb_error *err);

/* No reference counterpart: a host->device execution of a prepared template
 * that allocates nothing, for callers that cannot call cudaMalloc (code under
 * a caching allocator that owns the device heap, hosts with a fixed device
 * memory budget, code that must not allocate between graph captures). Instead
 * of a context's HBM ring and parameter buffers it uses one statically
 * allocated 32 MiB __device__ array (1 MiB of parameters, the rest one staging
 * slot for source rows) that every GPU loading libsb_cuda.so holds until exit.
 * `source` is host memory (pinned for full speed), `destination` device memory
 * of the template's destination size; all work is ordered on `stream` (NULL =
 * the legacy default stream) with no copy/compute overlap. Plans whose
 * parameters exceed 1 MiB, or whose single source row (or whole source, when
 * rows cannot be split) exceeds the staging slot, are rejected with
 * invalid_options. The scratch is the current device's: `destination` must
 * be memory of the current device (device_mismatch otherwise), and `stream`
 * a stream of it. The first call on a device resolves the array's device
 * address (cudaGetSymbolAddress) with that device current: make that first
 * call outside any stream capture. All calls share the array, so calls that
 * overlap on the GPU (other streams, other threads) race. Calls whose plan
 * checks its channel map on the device, or that ran a kernel with bounded
 * waits (the TMA tile transposes), synchronize `stream` before returning and
 * report a wait that ran out as backend_failure; otherwise the call returns
 * with the copies still queued on `stream`, and `source` must stay valid and
 * unchanged until `stream` has passed them. */
int sb_execute_h2d_static(const sb_template *tmpl, const void *source, void *destination, void *stream,
                          sb_error *err);

/* ---- consumer-sized groups and asynchronous completion ------------------- */
typedef struct sb_group sb_group;           /* a validated single-use group of requests */
typedef struct sb_completion sb_completion; /* a submitted group's pending completion */

/* One group member: a template (typed, or a layout plan's transfer
 * template) with fresh source/destination views. direction: 0 h2d. */
typedef struct {
  const sb_template *plan;
  sb_view source;
  sb_view destination;
  int32_t direction;
} sb_group_entry;

/* pyreloc.prepare_dispatch_group (PyDispatch.cpp:645; dispatch::
 * prepareDispatchGroup, Dispatch.h:213): validate 1..256 members together
 * (one device, no destination overlapping another destination or any source)
 * before anything is allocated or launched. */
int sb_prepare_dispatch_group(const sb_group_entry *entries, size_t count, sb_group **out, sb_error *err);
/* pyreloc.execute_dispatch_group (PyDispatch.cpp:648): every member after one
 * wait on the caller stream, one completion for all (blocking unless
 * options->async_completion). report: the group report JSON. */
int sb_execute_dispatch_group(sb_group *group, sb_resources *resources, const sb_options *options, char *report,
                              size_t cap, sb_error *err);
/* pyreloc.submit_dispatch_group (PyDispatch.cpp:696; Resources::submit,
 * DispatchResources.h:85): enqueue the group and return its completion
 * without waiting. resources may be NULL (a private context kept alive by the
 * completion). Source and destination buffers must stay valid until the
 * completion reports done. */
int sb_submit_dispatch_group(sb_group *group, sb_resources *resources, const sb_options *options,
                             sb_completion **out, sb_error *err);
/* The group report (totals and one report per member) as JSON. */
int sb_group_report(const sb_group *group, char *json, size_t cap);
void sb_group_free(sb_group *group);
/* DispatchCompletion.wait / query / wait_stream (PyDispatch.cpp:659-692). */
int sb_completion_wait(sb_completion *completion, sb_error *err);
/* *done = 1 once complete, 0 while pending. */
int sb_completion_query(sb_completion *completion, int32_t *done, sb_error *err);
/* Order `stream` (a cudaStream_t) after the group, without a host wait. */
int sb_completion_wait_stream(sb_completion *completion, void *stream, sb_error *err);
/* Releases the handle; waits for the group first if it is still pending. */
void sb_completion_free(sb_completion *completion);

/* pyreloc.DispatchResources (PyDispatch.cpp:700-801) / dispatch::Resources. */
int sb_resources_create(uint64_t max_retained_bytes, uint64_t max_live_bytes, uint32_t max_contexts,
                        sb_resources **out, sb_error *err);
int sb_resources_stats(const sb_resources *resources, char *json, size_t cap);
/* The copy-engine and compute streams (cudaStream_t) of the context of
 * `device`, created on first use; for callers that time or order work on them. */
int sb_resources_streams(sb_resources *resources, int32_t device, void **copy_stream, void **compute_stream,
                         sb_error *err);
/* Bound the wait for a context that another call holds (reference
 * DispatchResources acquireTimeoutMs, DispatchResources.h:70): after `ms`
 * milliseconds (0: at once) the call fails with acquire_timeout; a negative
 * value waits without limit (the default). */
void sb_resources_set_acquire_timeout(sb_resources *resources, int64_t ms);
int sb_resources_clear(sb_resources *resources, sb_error *err);
int sb_resources_close(sb_resources *resources, sb_error *err);
void sb_resources_free(sb_resources *resources);

#ifdef __cplusplus
}
#endif

#endif
