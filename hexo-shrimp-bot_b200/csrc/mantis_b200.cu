// Single translation unit of libmantis_b200.so: the kernels share one device
// error word, so they are compiled together.
#include "api.cu"
#include "tables.cu"
#include "rows.cu"
#include "attention.cu"
#include "radius.cu"
#include "gemm_simt.cu"
#include "gemm_sm100.cu"
#include "attention_sm100.cu"
#include "stone_sm100.cu"
#include "noalloc.cu"
#include "encoder.cu"
#include "klent.cu"
