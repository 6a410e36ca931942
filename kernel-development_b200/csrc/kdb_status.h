/* kdb_status.h — status codes shared by the host entry points and the device status word. */
#pragma once

#define KDB_OK 0
#define KDB_ERR_INVALID_ARG 1     /* bad size, null pointer, misaligned pointer or stride */
#define KDB_ERR_UNSUPPORTED 2     /* shape outside what the kernels implement */
#define KDB_ERR_CUDA 3            /* a CUDA runtime/driver call failed (see kdb_last_cuda_error) */
#define KDB_ERR_TIMEOUT 4         /* a bounded device wait gave up (device status word) */
#define KDB_ERR_WORKSPACE 5       /* workspace too small */
#define KDB_ERR_NO_DEVICE 6       /* no sm_100 device current */
#define KDB_ERR_DEVICE_BOUNDS 7   /* a kernel's own bounds check rejected an index (device status word) */
