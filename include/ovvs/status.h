#pragma once

/* Status codes returned by every ovvs entry point. The numeric values are ABI: bindings in
 * other languages hard-code them (reference include/ovvs/status.h:7-17). */

#ifdef __cplusplus
extern "C" {
#endif

typedef enum ovvsStatus {
  OVVS_STATUS_SUCCESS = 0,
  OVVS_STATUS_ERROR = 1,              /* CUDA/NCCL failure, kernel watchdog, internal error */
  OVVS_STATUS_INVALID_ARGUMENT = 2,   /* null pointer or non-positive size */
  OVVS_STATUS_UNSUPPORTED = 3,        /* entry point outside this library's scope */
  OVVS_STATUS_OOM = 4,                /* device or pinned-host allocation failed */
  OVVS_STATUS_COMPILE_FAIL = 5,       /* kept for ABI; never returned here */
  OVVS_STATUS_SHAPE_MISMATCH = 6,     /* sizes overflow the supported range */
  OVVS_STATUS_DEVICE_UNAVAILABLE = 7, /* no usable B200, or a CPU/NPU device was forced */
  OVVS_STATUS_IO = 8                  /* kept for ABI; never returned here */
} ovvsStatus;

#ifdef __cplusplus
}
#endif
