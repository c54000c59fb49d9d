// Debug-bounds build of ../gdn_tc.cu: the same source compiled with BDLLM_DEBUG_BOUNDS
// (index, alignment and non-finite checks; records read by bounds_report()).
#define BDLLM_DEBUG_BOUNDS 1
#include "../gdn_tc.cu"
