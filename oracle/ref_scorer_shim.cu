// Test-only C entry point around the reference's own decode scorer.
//
// Test infrastructure: oracle/build_ref_cuda.py compiles this file together
// with the reference source `library/AdaptiveIMI/cpp_extensions/cuda/
// compute_impl.cu`, read in place from the reference checkout, into
// `oracle/_ref/libref_scorer.so`.  Only the GPU pin test loads it; the product
// never does.  The declaration below is the one the reference's own wrapper
// uses (compute_wrappers.cpp:13-22); this shim only drops the torch tensors.
#include <cuda_runtime.h>

namespace imi_decode {
void fused_query_group_similarities_bf16(const void* query_grouped, const float* centroids, float* similarities,
                                         int num_query_groups, int n_clusters, int kv_heads, int dim,
                                         cudaStream_t stream);
}

extern "C" int ref_fused_query_group_similarities_bf16(const void* q, const float* centroids, float* out, int groups,
                                                       int n_clusters, int kv_heads, int dim, void* stream) {
    imi_decode::fused_query_group_similarities_bf16(q, centroids, out, groups, n_clusters, kv_heads, dim,
                                                    static_cast<cudaStream_t>(stream));
    return static_cast<int>(cudaGetLastError());
}
