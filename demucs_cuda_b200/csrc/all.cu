// Single translation unit of libdc_b200.so: the parts below share file-local state (the
// backend stream, the device fault word, scratch buffers) without relocatable device code.
#include "runtime.cu"
#include "trace.cu"
#include "elementwise.cu"
#include "norm.cu"
#include "operand.cu"
#include "spectral.cu"
#include "gemm.cu"
#include "attention.cu"
#include "glue.cu"
#include "engine.cu"
#include "forward.cu"
