// Internal to sym_b200: the statically allocated device scratch behind
// sb_execute_h2d_static (include/sym_b200.h). Not part of the public C-ABI.
#ifndef SYM_B200_STATIC_SCRATCH_H
#define SYM_B200_STATIC_SCRATCH_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/// Size of the file-scope device array every GPU that loads libsb_cuda.so
/// holds until process exit.
#define SBC_STATIC_SCRATCH_BYTES (32u << 20)

/// Device address of the static scratch on the current device. The first
/// call on a device resolves it with cudaGetSymbolAddress (that device made
/// current by the caller) and caches it; later calls only read the cache.
/// Returns a cudaError_t status; allocates nothing.
int sbc_static_scratch(void **device_ptr, size_t *bytes);

#ifdef __cplusplus
}
#endif

#endif
