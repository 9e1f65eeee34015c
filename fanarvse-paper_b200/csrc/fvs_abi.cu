// Library identification entry points.
#include "fvs_common.cuh"

extern "C" int fvs_version(void) { return 100; }
extern "C" const char* fvs_arch(void) { return "sm_100a"; }
