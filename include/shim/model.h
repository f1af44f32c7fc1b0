/* Shim for relinking a reference caller (src/main.c and friends) against
 * libqwenb200: the reference's gguf.h / threadpool.h keep providing the shared
 * types, and the model / kernel API resolves to include/qwen_b200.h.  Put this
 * directory first on the include path (-Iinclude/shim -I<reference>/include
 * -Iinclude). */
#ifndef QWEN_B200_SHIM_MODEL_H
#define QWEN_B200_SHIM_MODEL_H
#include "gguf.h"
#include "threadpool.h"
#include "sampler.h"
#include "qwen_b200.h"
#endif
