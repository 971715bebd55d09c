// imi_internal.h -- kernel argument blocks and launchers shared by the .cu
// files and the C-ABI layer (capi.cpp).  Not part of the public interface.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <string>
#include <utility>

#include "../../include/imi_b200.h"

namespace imi {

using SelectArgs = imi_select_desc;
using AttnArgs = imi_attn_desc;
using AppendArgs = imi_append_desc;
using AsyncArgs = imi_async_desc;
using ApplyArgs = imi_apply_desc;
using BuildArgs = imi_build_desc;
using MergeArgs = imi_merge_desc;
using CombineArgs = imi_combine_desc;
using PeerGatherArgs = imi_peer_gather_desc;

cudaError_t launch_similarity(const uint16_t* q, const float* cent, float* out, int bg, int G, int n_cells, int dim,
                              long long out_stride, cudaStream_t st);
size_t select_smem_bytes(const SelectArgs& a);
int select_max_slots();
// app: when given, the select kernel also performs that steady-zone append
// (for the same groups), in place of a separate append launch.
cudaError_t launch_select(const SelectArgs& a, cudaStream_t st, const AppendArgs* app = nullptr);
size_t attn_smem_bytes(const AttnArgs& a);
cudaError_t launch_attention(const AttnArgs& a, cudaStream_t st);
size_t merge_smem_bytes(const MergeArgs& a);
cudaError_t launch_merge(const MergeArgs& a, cudaStream_t st);
cudaError_t launch_combine_shards(const CombineArgs& a, cudaStream_t st);
cudaError_t launch_peer_allgather(const PeerGatherArgs& a, cudaStream_t st);
cudaError_t launch_append(const AppendArgs& a, cudaStream_t st);
size_t async_smem_bytes(const AsyncArgs& a);
cudaError_t launch_async_assign(const AsyncArgs& a, cudaStream_t st);
int async_chunks(int n_slots);
cudaError_t launch_apply(const ApplyArgs& a, cudaStream_t st);

size_t build_workspace_bytes(int heads, int n, int dim, int parts, const int* ks);
void set_last_error(const std::string& msg);
cudaError_t ensure_smem(const void* func, size_t bytes, int* cache, int cache_len);

#ifdef __CUDACC__
// Steady-zone append of group h: warp t (0 keys, 1 values) copies the new row
// into zone[h, pos] and, when given, the async-update batch slot
// (runtime.py:378-392, async_update.py:115-117).
__device__ inline void append_group(const AppendArgs& a, int h, int t, int lane) {
    const uint4* src = reinterpret_cast<const uint4*>(
        reinterpret_cast<const unsigned char*>(t ? a.new_values : a.new_keys) + (size_t)h * a.src_head_stride * 2);
    uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<unsigned char*>(t ? a.zone_values : a.zone_keys) +
                                          ((size_t)h * a.zone_rows + a.pos) * a.dim * 2);
    const int n16 = a.dim * 2 / 16;
    for (int i = lane; i < n16; i += 32) {
        const uint4 v = src[i];
        dst[i] = v;
        if (a.batch_keys) {
            uint4* bd = reinterpret_cast<uint4*>(reinterpret_cast<unsigned char*>(t ? a.batch_values : a.batch_keys) +
                                                 ((size_t)h * a.batch_cap + a.batch_slot) * a.dim * 2);
            bd[i] = v;
        }
    }
}
#endif

// Programmatic dependent launch: the kernel may be scheduled while the kernel
// before it in the stream is still running (once that one has executed
// griddepcontrol.launch_dependents or finished); it must execute
// griddepcontrol.wait before touching memory the earlier kernels write.
template <typename... Params, typename... Args>
cudaError_t launch_pdl(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                       Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}
cudaError_t run_build(const BuildArgs& a, cudaStream_t st, const char** why);


}  // namespace imi
