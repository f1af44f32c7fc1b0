/* Shim: the reference kernels.h API (gemv_*, rmsnorm, ...) from libqwenb200.
 * See include/shim/model.h. */
#ifndef QWEN_B200_SHIM_KERNELS_H
#define QWEN_B200_SHIM_KERNELS_H
#include "model.h"
#endif
