// Shared helpers for the swarmlora_b200 C-ABI library: status codes, the
// thread-local "last error" string every entry point fills on failure, and
// CUDA error-check macros that turn a failing call into a status return.
//
// Error convention: every extern "C" entry point returns an int status
// (SWL_OK == 0, negative on failure) and leaves a human-readable message in
// swl_last_error(). The Python modules raise RuntimeError(message), which is
// what the reference's pybind modules do when their C++ throws
// std::runtime_error (ipc_types.h:223-229 CUDA_RT_CHECK).
#pragma once

#include <cstddef>
#include <cstdint>
#include <cstdio>
#include <cstdarg>
#include <string>
#include <cuda_runtime.h>

#define SWL_OK 0
#define SWL_ERR_ARG -1        // invalid argument / API misuse
#define SWL_ERR_STATE -2      // called in the wrong state (not initialised ...)
#define SWL_ERR_CUDA -3       // a CUDA runtime / driver call failed
#define SWL_ERR_SYS -4        // an OS call (shm_open, mmap ...) failed
#define SWL_ERR_FULL -5       // ring buffer full / no free slot
#define SWL_ERR_QUIT -6       // quit flag observed while waiting
#define SWL_ERR_TIMEOUT -7    // a bounded wait ran out
#define SWL_ERR_OWNER -8      // slot ownership check failed

namespace swl {

// Sets the calling thread's last-error message and returns `code`.
int set_error(int code, const char* fmt, ...);
const char* last_error();
// The device allocation holding `p` (its base and size); defined with the
// aggregator's allocation bookkeeping.
int allocation_of(const void* p, char** base, size_t* size);

}  // namespace swl

#define SWL_CUDA_TRY(call)                                                      \
  do {                                                                          \
    cudaError_t _e = (call);                                                    \
    if (_e != cudaSuccess) {                                                    \
      return swl::set_error(SWL_ERR_CUDA, "CUDA error: %s (%s:%d: %s)",         \
                            cudaGetErrorString(_e), __FILE__, __LINE__, #call); \
    }                                                                           \
  } while (0)

#define SWL_TRY(expr)          \
  do {                         \
    int _s = (expr);           \
    if (_s != SWL_OK) return _s; \
  } while (0)

#define SWL_EXPORT extern "C" __attribute__((visibility("default")))
