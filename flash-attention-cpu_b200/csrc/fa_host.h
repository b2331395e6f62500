// Internal interface between the C ABI (fa_capi.cu) and the multi-device
// orchestration of the host-slice calls (fa_devices.cu).  Not exported.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>

#include <string>

#include "fa_common.cuh"

namespace fa {
// fa_capi.cu: the calling thread's error message and status codes.
int status_error(int code, const std::string& msg);
int status_cuda(cudaError_t e, const char* what);
std::string status_message();
// Makes `dev` current and initialises the library's state on it.
int prepare_device_on(int dev);
int device_sm_count(int dev);
// Kernel selection and launch of one forward on device `dev` (current).
int dispatch_on(FwdParams p, int dev, cudaStream_t s);
// Waits for `s`, then reads and clears the device's bounded-wait error word.
int check_err_flag_on(int dev, cudaStream_t s);
// The whole host-slice forward on one device (copies in, kernels, copies out).
int host_forward_on(int dev, const float* q, const float* k, const float* v, size_t bh,
                    size_t sq, size_t sk, size_t d, int causal, float* out, float* lse);

// fa_devices.cu: the host-slice forward over a list of devices.
int host_forward_devices(const int* devs, int n, const float* q, const float* k, const float* v,
                         size_t bh, size_t sq, size_t sk, size_t d, int causal, float* out,
                         float* lse);
// Frees the cached streams, events and workspaces of the multi-device path.
void devices_release();
}  // namespace fa
