// Per-head kernel instantiations for element type __half.
#include "heads_inst.cuh"

BLOTH_INSTANTIATE_HEADS(__half)
