// Tensor-core (tcgen05) path of the fused attention -- placeholder until the
// sm_100a kernel lands; every shape is served by the CUDA-core path meanwhile.
#include "sas_common.cuh"

namespace sas_host {

bool tc_supported(const SasFwdArgs &) { return false; }
size_t tc_workspace(const SasFwdArgs &) { return 0; }
int launch_fwd_tc(const SasFwdArgs &, const sas::FwdLayout &, char *, const void *, const void *, const int32_t *,
                  const void *, const float *, void *, float *, cudaStream_t) {
    return SAS_ERR_UNSUPPORTED;
}

} // namespace sas_host
