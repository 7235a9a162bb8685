/*
 * orc_ops.c -- CPU oracle for the fused ops on the GEMM path. TEST INFRASTRUCTURE ONLY.
 * (filled in op by op; each function cites the reference lines it restates)
 */
#include <math.h>
#include <stddef.h>
