// Per-head kernel instantiations for element type __nv_bfloat16.
#include "heads_inst.cuh"

BLOTH_INSTANTIATE_HEADS(__nv_bfloat16)
