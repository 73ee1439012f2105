/* vgpu_npu.h - legacy include name of the vgpu_npu_* API (reference
 * include/vgpu_npu.h); the declarations are in vnpu_compat.h. */
#ifndef VNPU_B200_VGPU_NPU_H
#define VNPU_B200_VGPU_NPU_H
#include "vnpu_compat.h"
#endif
