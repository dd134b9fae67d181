// Row-kernel instantiations for element type __nv_bfloat16.
#include "rows_inst.cuh"

BLOTH_INSTANTIATE_ROWS(__nv_bfloat16)
