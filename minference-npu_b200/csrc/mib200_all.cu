// Single translation unit for libminference_b200.so, so device globals
// (the error word) are shared without relocatable device code.
#include "capi.cu"
#include "attention.cu"
#include "block_sparse.cu"
#include "vs_index.cu"
#include "noalloc.cu"
