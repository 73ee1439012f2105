/* includes/private/video/vgpu_npu.h - the emulator-era include path of the
 * vgpu_npu_* API (reference include/includes/private/video/vgpu_npu.h).
 * Compile with -I<include> so vnpu_compat.h resolves. */
#ifndef VNPU_B200_PRIVATE_VIDEO_VGPU_NPU_H
#define VNPU_B200_PRIVATE_VIDEO_VGPU_NPU_H
#include "vnpu_compat.h"
#endif
