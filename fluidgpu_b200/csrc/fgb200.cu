// Single translation unit of libfgb200.so: every component is included here
// so device globals (the status word) and helpers need no separate device link.
#include "common.cuh"
#include "runtime.cuh"
#include "elementwise.cuh"
#include "gemm.cuh"
#include "attention.cuh"
#include "attention_noalloc.cuh"
#include "moe.cuh"
#include "handoff.cuh"
#include "disagg.cuh"
