// The bounds-checked build of attn/attention_bwd.cu (compiled with -DH3_BOUNDS_CHECK into
// h3_a100._C_checked; a separate file so its objects do not collide with the
// normal build's).
#include "../attn/attention_bwd.cu"
