// moe_rows.cu compiled with the bounds checks on (module mamformer_b200._C_check).
#define MAMF_BOUNDS_CHECK 1
#include "../moe_rows.cu"
