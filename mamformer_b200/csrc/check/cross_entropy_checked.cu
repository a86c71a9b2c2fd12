// cross_entropy.cu compiled with the bounds checks on (module mamformer_b200._C_check).
#define MAMF_BOUNDS_CHECK 1
#include "../cross_entropy.cu"
