// host_common.h -- host-side helpers shared by the C-ABI entry points: the thread-local error
// string behind tokmix_last_error(), status codes, and TMA tensor-map encoding through the
// driver entry point (so the library links only against the CUDA runtime).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <mutex>
#include <string>

#include "../../include/tokmix.h"

namespace tokmix {

void set_error(const char* fmt, ...);

// Records the error and returns the status code, for `return fail(TOKMIX_ERR_..., "...")`.
int fail(int code, const char* fmt, ...);

// Checks the result of a launch (cudaGetLastError) and maps it to a status code.
int check_launch(const char* what);

// TMA tiled tensor map over a tensor of `rank` dims (dims[0] innermost), element type dt.
// strides_bytes has rank-1 entries (byte strides of dims 1..rank-1).  Returns false (and sets
// the error string) if the driver rejects the encoding.
bool encode_tiled(CUtensorMap* map, CUtensorMapDataType dt, int rank, const void* base, const uint64_t* dims,
                  const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swizzle);

// Number of SMs of the current device.
int device_sm_count();

// Sets the dynamic shared memory limit of a kernel once per (kernel, device, size).
bool ensure_smem_attr(const void* func, int bytes);

// TOKMIX_OK if the current device is a compute capability 10.0 part, else sets the error.
int check_device();

// The GDN stage-1 options (tokmix_gdn_stage1): whether gates / q-k normalisation are requested,
// and their checks -- gates need a, b, a_log, dt_bias and a bf16 or fp32 dtype; normalisation a
// positive finite eps and, for the schedules that need it, the normalised-key buffer.
inline bool stage1_gates(const tokmix_gdn_stage1* s1) { return s1 != nullptr && s1->a != nullptr; }
inline bool stage1_l2norm(const tokmix_gdn_stage1* s1) { return s1 != nullptr && s1->qk_l2norm != 0; }
int check_stage1(const char* who, const tokmix_gdn_stage1* s1, bool needs_k_normed);

}  // namespace tokmix
