// Address-space switch for host compilation of the reference kernels.
#undef threadgroup
#define threadgroup
#include_next "radix_sort.metal.h"
