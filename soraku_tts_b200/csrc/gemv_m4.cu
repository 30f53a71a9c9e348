#define GEMV_M 4
#include "gemv_inst.cuh"
