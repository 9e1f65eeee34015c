// Library identification entry points and the wait-limit knob of the tcgen05 kernels.
#include <atomic>

#include "fvs_common.cuh"
#include "fvs_tcgen05.cuh"

extern "C" int fvs_version(void) { return 100; }
extern "C" const char* fvs_arch(void) { return "sm_100a"; }

// Pipeline wait limit of the tcgen05 kernels, passed to each launch as an argument.
static_assert(FVS_WAIT_LIMIT_DEFAULT == fvs::tcg::WAIT_LIMIT, "header and kernels agree on the default limit");
static std::atomic<uint32_t> g_wait_limit{fvs::tcg::WAIT_LIMIT};

uint32_t fvs::tcg::pipeline_wait_limit() { return g_wait_limit.load(std::memory_order_relaxed); }

extern "C" uint32_t fvs_set_wait_limit(uint32_t polls) { return g_wait_limit.exchange(polls); }
