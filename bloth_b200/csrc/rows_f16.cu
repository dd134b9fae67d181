// Row-kernel instantiations for element type __half.
#include "rows_inst.cuh"

BLOTH_INSTANTIATE_ROWS(__half)
