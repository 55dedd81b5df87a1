// vxc_internal.h — host-side declarations shared by the library's .cu files.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>
#include "../../include/veltrix_cuda.h"

void vxc_set_error(const char *fmt, ...);
// 0 when a CUDA device is current; VX_ERR_UNSUPPORTED otherwise.
int vxc_require_device(void);
// Per-device error word (device memory), valid after vxc_require_device().
unsigned int *vxc_device_error_ptr(void);
int vxc_launch_splitk_reduce(const float *ws, int ks, int M, int R, float *y, cudaStream_t st);
size_t vxc_qgemv_simt_ws(const vxc_qmat *w, int M);
// Library-wide count of kernel launches (a CUDA-graph replay adds its kernels).
void vxc_count_launches(long long n);
