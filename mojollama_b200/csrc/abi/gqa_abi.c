/* Reference-named entry point of gqa_attention.so
 * (src/mojollama/kernels/gqa_attention.c of the reference), forwarding to
 * libmojollama_b200.so. */
#include "mojollama_b200.h"
