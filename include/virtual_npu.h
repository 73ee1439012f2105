/* virtual_npu.h - legacy include name of the virtual_npu_* API (reference
 * include/virtual_npu.h); the declarations are in vnpu_compat.h. */
#ifndef VNPU_B200_VIRTUAL_NPU_H
#define VNPU_B200_VIRTUAL_NPU_H
#include "vnpu_compat.h"
#endif
