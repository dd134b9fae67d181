// Row-kernel instantiations for element type float.
#include "rows_inst.cuh"

BLOTH_INSTANTIATE_ROWS(float)
