// tcgen05 / TMEM / TMA attention kernels (sm_100a).  Placeholder: the
// tensor-core path is not enabled yet, so no configuration is eligible.
#include "common.cuh"

bool scope_tc_eligible(const ScopeAttnArgs &, bool) { return false; }
int scope_tc_fwd(const ScopeAttnArgs &, cudaStream_t) { return SCOPE_ERR_UNSUPPORTED; }
int scope_tc_bwd(const ScopeAttnArgs &, cudaStream_t) { return SCOPE_ERR_UNSUPPORTED; }
