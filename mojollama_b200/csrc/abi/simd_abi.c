/* Reference-named entry points of simd_ops.so (src/mojollama/kernels/simd_ops.c of
 * the reference), forwarding to libmojollama_b200.so. */
#include "mojollama_b200.h"

void set_num_threads(int n) { (void)n; }
