// lib.cu — single translation unit of libspectral_b200.so (the device status
// word and the kernels share one module).
#include <vector>
#include "common.cu"
#include "router.cu"
#include "ternary.cu"
#include "enhanced.cu"
#include "pipeline.cu"
#include "tree.cu"
#include "gas.cu"
#include "ep.cu"
