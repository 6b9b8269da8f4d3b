// Tensor-core attention path (placeholder until the tcgen05 kernel lands).
#include "tc.cuh"

namespace mla {

bool tc_attention_supported(const AArgs&) { return false; }
template <typename T> size_t tc_attention_workspace(const AArgs&) { return 0; }
template <typename T> mla_status_t tc_attention(const AArgs&, cudaStream_t) {
    return set_error(MLA_ERR_UNSUPPORTED, "MLA: tensor-core attention not built");
}
template size_t tc_attention_workspace<float>(const AArgs&);
template size_t tc_attention_workspace<double>(const AArgs&);
template size_t tc_attention_workspace<__half>(const AArgs&);
template size_t tc_attention_workspace<__nv_bfloat16>(const AArgs&);
template mla_status_t tc_attention<float>(const AArgs&, cudaStream_t);
template mla_status_t tc_attention<double>(const AArgs&, cudaStream_t);
template mla_status_t tc_attention<__half>(const AArgs&, cudaStream_t);
template mla_status_t tc_attention<__nv_bfloat16>(const AArgs&, cudaStream_t);

}  // namespace mla
