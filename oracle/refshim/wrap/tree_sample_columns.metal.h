// Address-space switch for host compilation of the reference kernels.
#undef threadgroup
#define threadgroup volatile
#include_next "tree_sample_columns.metal.h"
