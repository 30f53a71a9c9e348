#define GEMV_M 1
#include "gemv_inst.cuh"
