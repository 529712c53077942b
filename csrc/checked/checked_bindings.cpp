// The bounds-checked build of the bindings (module h3_a100._C_checked).
#include "../bindings.cpp"
