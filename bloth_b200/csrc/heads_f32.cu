// Per-head kernel instantiations for element type float.
#include "heads_inst.cuh"

BLOTH_INSTANTIATE_HEADS(float)
