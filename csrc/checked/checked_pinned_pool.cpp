// The bounds-checked build of the pinned staging pool (module h3_a100._C_checked).
#include "../staging/pinned_pool.cpp"
