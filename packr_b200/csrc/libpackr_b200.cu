// Single translation unit of libpackr_b200.so: every kernel and every C-ABI
// entry point is compiled together so that device globals are shared without
// relocatable device code.
#include "common.cu"
#include "adam8.cu"
#include "prep.cu"
#include "gemm.cu"
#include "predecode.cu"
#include "gemv.cu"
#include "skinny.cu"
#include "linear.cu"
#include "static_scratch.cu"
#include "velvet.cu"
#include "compress.cu"
#include "peer.cu"
