// gpu_spmv.cuh -- umbrella of the GPU SpMV operators
// (structural/include/structural/gpu_spmv.cuh): the per-codec operator
// wrappers and run_bitbsr_spmv_once.
#pragma once

#include "structural/operators/bitbsr_spmv_8x4.cuh"
#include "structural/operators/bitbsr_spmv_8x4_dispatch.cuh"
