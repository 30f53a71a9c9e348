#define GEMV_M 2
#include "gemv_inst.cuh"
