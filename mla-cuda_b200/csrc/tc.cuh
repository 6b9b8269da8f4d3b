// Tensor-core (tcgen05) attention path: MLA_PREC_TENSOR, and MLA_PREC_EXACT for
// 16-bit storage (exact = true: fp32 partial scores and a two-part P, so the
// arithmetic is the reference's fp32-accumulate policy for 16-bit storage).
#pragma once

#include "qprep.cuh"

namespace mla {

// True when the tensor-core kernel covers this shape (otherwise the exact
// path runs).
bool tc_attention_supported(const AArgs& a);
template <typename T> size_t tc_attention_workspace(const AArgs& a);
template <typename T> mla_status_t tc_attention(const AArgs& a, cudaStream_t st, bool exact = false);

}  // namespace mla
