// capi.cu -- the extern "C" entry points declared in include/imi_b200.h.
// Validation, error reporting (thread-local last error) and dispatch to the
// kernel launchers.  No entry point allocates device memory.
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>
#include <string>

#include "imi_internal.h"

namespace {

thread_local std::string g_last_error;

int fail(int code, const std::string& msg) {
    g_last_error = msg;
    return code;
}

int cuda_status(cudaError_t e, const char* where) {
    if (e == cudaSuccess) return IMI_OK;
    return fail(IMI_ERR_CUDA, std::string(where) + ": " + cudaGetErrorString(e));
}

inline cudaStream_t S(void* s) { return static_cast<cudaStream_t>(s); }

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

namespace imi {
void set_last_error(const std::string& msg) { g_last_error = msg; }

// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) once per device and size:
// `cache` holds the largest size already set on each device.
cudaError_t ensure_smem(const void* func, size_t bytes, int* cache, int cache_len) {
    static std::mutex mu;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lock(mu);
    if (dev >= 0 && dev < cache_len && (int)bytes <= cache[dev]) return cudaSuccess;
    e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e == cudaSuccess && dev >= 0 && dev < cache_len) cache[dev] = (int)bytes;
    return e;
}
}  // namespace imi

extern "C" {

int imi_abi_version(void) { return IMI_ABI_VERSION; }

const char* imi_last_error(void) { return g_last_error.c_str(); }

size_t imi_build_workspace_size(int32_t heads, int32_t n_tokens, int32_t dim, int32_t parts, const int32_t* ks) {
    if (!ks || heads <= 0 || n_tokens <= 0) return 0;
    return imi::build_workspace_bytes(heads, n_tokens, dim, parts, ks);
}

int imi_build_index(const imi_build_desc* d, void* stream) {
    if (!d) return fail(IMI_ERR_INVALID, "imi_build_index: null descriptor");
    if (!d->keys || !d->values || !d->list_keys || !d->list_values || !d->cell_sizes || !d->cell_offsets ||
        !d->cell_mask || !d->cell_code || !d->centroids || !d->sub_centroids || !d->n_active)
        return fail(IMI_ERR_INVALID, "imi_build_index: null pointer in descriptor");
    if (d->heads <= 0) return fail(IMI_ERR_INVALID, "imi_build_index: heads must be positive");
    if (d->list_rows < d->n_tokens) return fail(IMI_ERR_INVALID, "imi_build_index: list_rows < n_tokens");
    if (d->n_slots < 1) return fail(IMI_ERR_INVALID, "imi_build_index: n_slots must be positive");
    const char* why = "";
    cudaError_t e = imi::run_build(*d, S(stream), &why);
    if (e == cudaErrorInvalidValue && why[0]) return fail(IMI_ERR_INVALID, std::string("imi_build_index: ") + why);
    return cuda_status(e, "imi_build_index");
}

int imi_query_group_similarities(const uint16_t* q, const float* centroids, float* out, int32_t kv_heads,
                                 int32_t groups, int32_t n_clusters, int32_t dim, int64_t out_stride, void* stream) {
    if (!q || !centroids || !out) return fail(IMI_ERR_INVALID, "imi_query_group_similarities: null pointer");
    if (kv_heads <= 0 || groups <= 0 || n_clusters < 0 || dim <= 0 || dim % 4 != 0)
        return fail(IMI_ERR_INVALID, "imi_query_group_similarities: bad shape");
    if (out_stride < n_clusters) return fail(IMI_ERR_INVALID, "imi_query_group_similarities: out_stride < n_clusters");
    if (!aligned16(centroids)) return fail(IMI_ERR_INVALID, "imi_query_group_similarities: centroids not 16-byte aligned");
    if (n_clusters == 0) return IMI_OK;
    return cuda_status(imi::launch_similarity(q, centroids, out, kv_heads, groups, n_clusters, dim, out_stride, S(stream)),
                       "imi_query_group_similarities");
}

static int check_select(const imi_select_desc* d) {
    if (!d) return fail(IMI_ERR_INVALID, "imi_select_cells: null descriptor");
    const int Sp = d->parts == 0 ? 1 : d->parts;
    if (!(d->parts == 0 || d->parts == 2 || d->parts == 4) || d->dim != 128)
        return fail(IMI_ERR_INVALID, "imi_select_cells: parts must be 0/2/4 and dim 128");
    if (d->bg <= 0 || d->G <= 0 || d->n_slots <= 0 || d->nprobe <= 0 || d->page_size <= 0)
        return fail(IMI_ERR_INVALID, "imi_select_cells: bad sizes");
    if (!d->q || !d->cell_code || !d->cell_sizes || !d->cell_offsets || !d->cell_mask || !d->centroids ||
        !d->sub_centroids || !d->sel_cells || !d->sel_count || (!d->row_index != !d->row_count))
        return fail(IMI_ERR_INVALID, "imi_select_cells: null pointer in descriptor");
    if (d->nprobe > imi::select_max_slots())
        return fail(IMI_ERR_INVALID, "imi_select_cells: nprobe > " + std::to_string(imi::select_max_slots()) + " is not supported");
    if (d->key_base < 0 || (int64_t)d->key_base + d->n_slots > 0x7fffffffLL)
        return fail(IMI_ERR_INVALID, "imi_select_cells: key_base + n_slots must fit in 31 bits");
    if (d->static_len < 0 || d->static_len + (int64_t)d->buffer_pages * d->page_size > d->exec_capacity)
        return fail(IMI_ERR_INVALID, "imi_select_cells: exec_capacity < static_len + buffer_pages*page_size");
    long long table = 1;
    for (int s = 0; s < Sp; ++s) {
        if (d->ks[s] < 1 || d->ks[s] > d->kmax || (Sp > 1 && d->ks[s] > 255))
            return fail(IMI_ERR_INVALID, "imi_select_cells: bad k per subspace");
        if (s < Sp - 1) table *= d->ks[s];
    }
    if (table > 8192) return fail(IMI_ERR_INVALID, "imi_select_cells: prefix table (product of the first S-1 k) > 8192");
    if (d->delta_count && (!d->delta_cell_ids || d->delta_capacity <= 0))
        return fail(IMI_ERR_INVALID, "imi_select_cells: delta ring needs ids and capacity");
    if (d->n_slots > imi::select_max_slots())
        return fail(IMI_ERR_INVALID, "imi_select_cells: n_slots > " + std::to_string(imi::select_max_slots()));
    const size_t sm = imi::select_smem_bytes(*d);
    if (sm > 227 * 1024)
        return fail(IMI_ERR_INVALID, "imi_select_cells: n_slots too large for the on-chip selection (" +
                                         std::to_string(sm) + " bytes of shared memory)");
    return IMI_OK;
}

static int check_attention(const imi_attn_desc* d) {
    if (!d) return fail(IMI_ERR_INVALID, "imi_sparse_attention: null descriptor");
    if (d->bg <= 0 || d->G <= 0 || d->G > 8 || d->splits <= 0 || d->splits > 4096 || d->splits * d->G > 16384)
        return fail(IMI_ERR_INVALID, "imi_sparse_attention: need 1 <= G <= 8, 1 <= splits <= 4096, splits * G <= 16384");
    if (!d->q || !d->row_index || !d->row_count || !d->list_keys || !d->list_values || !d->static_keys ||
        !d->static_values || !d->part_o || !d->part_ml || (!d->out && !d->o_part))
        return fail(IMI_ERR_INVALID, "imi_sparse_attention: null pointer in descriptor");
    if ((d->o_part || d->ml_part) && (!d->o_part || !d->ml_part || !d->counters || !aligned16(d->o_part) ||
                                      (reinterpret_cast<uintptr_t>(d->ml_part) & 7u) != 0))
        return fail(IMI_ERR_INVALID,
                    "imi_sparse_attention: o_part and ml_part go together, need counters, and must be 16/8-byte aligned");
    if (!aligned16(d->list_keys) || !aligned16(d->list_values) || !aligned16(d->static_keys) ||
        !aligned16(d->static_values) || !aligned16(d->q))
        return fail(IMI_ERR_INVALID, "imi_sparse_attention: K/V/q buffers must be 16-byte aligned");
    if (!aligned16(d->part_o) || (reinterpret_cast<uintptr_t>(d->part_ml) & 7u) != 0 ||
        (reinterpret_cast<uintptr_t>(d->out) & 7u) != 0)
        return fail(IMI_ERR_INVALID, "imi_sparse_attention: part_o must be 16-byte and part_ml/out 8-byte aligned");
    if (d->exec_capacity <= 0) return fail(IMI_ERR_INVALID, "imi_sparse_attention: exec_capacity must be positive");
    return IMI_OK;
}

static int check_append(const imi_append_desc* d) {
    if (!d || !d->new_keys || !d->new_values || !d->zone_keys || !d->zone_values)
        return fail(IMI_ERR_INVALID, "imi_decode_append: null pointer");
    if (d->bg <= 0 || d->dim <= 0 || (d->dim * 2) % 16 != 0 || d->pos < 0 || d->pos >= d->zone_rows)
        return fail(IMI_ERR_INVALID, "imi_decode_append: position outside the steady zone");
    if (d->batch_keys && (d->batch_slot < 0 || d->batch_slot >= d->batch_cap))
        return fail(IMI_ERR_INVALID, "imi_decode_append: batch slot out of range");
    if (!aligned16(d->new_keys) || !aligned16(d->new_values) || (d->src_head_stride * 2) % 16 != 0)
        return fail(IMI_ERR_INVALID, "imi_decode_append: new k/v must be 16-byte aligned");
        return IMI_OK;
}

static int check_async(const imi_async_desc* d) {
    if (!d || !d->batch_keys || !d->batch_values || !d->sub_centroids || !d->cell_code || !d->shadow ||
        !d->counts || !d->delta_counts || !d->delta_sums || !d->ring_keys || !d->ring_values || !d->ring_cell_ids ||
        !d->ring_write_pos || !d->ring_count)
        return fail(IMI_ERR_INVALID, "imi_async_assign: null pointer");
    if (d->batch <= 0 || d->batch > d->batch_cap || d->batch > 64 || d->ring_cap <= 0 || d->dim != 128)
        return fail(IMI_ERR_INVALID, "imi_async_assign: bad batch / ring sizes");
    if (!d->part_best || d->part_chunks != imi::async_chunks(d->n_slots))
        return fail(IMI_ERR_INVALID, "imi_async_assign: part_best scratch with part_chunks = ceil(n_slots/512) required");
    if (imi::async_smem_bytes(*d) > 227 * 1024) return fail(IMI_ERR_INVALID, "imi_async_assign: batch too large");
    {
        const int Sp = d->parts == 0 ? 1 : d->parts;
        long long table = 1;
        for (int s = 0; s < Sp - 1; ++s) table *= d->ks[s];
        if (table * d->batch > 16384 || table * d->batch > 32 * 512)
            return fail(IMI_ERR_INVALID, "imi_async_assign: batch * prefix table > 16384");
    }
        return IMI_OK;
}

int imi_select_cells(const imi_select_desc* d, void* stream) {
    const int st = check_select(d);
    if (st != IMI_OK) return st;
    return cuda_status(imi::launch_select(*d, S(stream)), "imi_select_cells");
}

int imi_sparse_attention(const imi_attn_desc* d, void* stream) {
    const int st = check_attention(d);
    if (st != IMI_OK) return st;
    return cuda_status(imi::launch_attention(*d, S(stream)), "imi_sparse_attention");
}

static int check_decode_attend(const imi_select_desc* sel, const imi_attn_desc* attn, const imi_apply_desc* apply) {
    int st = check_select(sel);
    if (st != IMI_OK) return st;
    st = check_attention(attn);
    if (st != IMI_OK) return st;
    if (sel->bg != attn->bg || sel->G != attn->G || sel->row_index != attn->row_index ||
        sel->row_count != attn->row_count || sel->q != attn->q || sel->exec_capacity != attn->exec_capacity)
        return fail(IMI_ERR_INVALID, "imi_decode_attend: select and attention descriptors disagree");
    if (apply && (!apply->shadow || !apply->live || !apply->pending || !apply->live_dirty))
        return fail(IMI_ERR_INVALID, "imi_decode_attend: null pointer in apply descriptor");
    return IMI_OK;
}

// app: a steady-zone append that the select kernel performs itself
static int launch_decode_attend(const imi_select_desc* sel, const imi_attn_desc* attn, const imi_apply_desc* apply,
                                void* stream, const imi_append_desc* app = nullptr) {
    if (apply) {
        cudaError_t e = imi::launch_apply(*apply, S(stream));
        if (e != cudaSuccess) return cuda_status(e, "imi_decode_attend(apply)");
    }
    cudaError_t e = imi::launch_select(*sel, S(stream), app);
    if (e != cudaSuccess) return cuda_status(e, "imi_decode_attend(select)");
    return cuda_status(imi::launch_attention(*attn, S(stream)), "imi_decode_attend(attention)");
}


int imi_decode_attend(const imi_select_desc* sel, const imi_attn_desc* attn, const imi_apply_desc* apply,
                      void* stream) {
    const int st = check_decode_attend(sel, attn, apply);
    if (st != IMI_OK) return st;
    return launch_decode_attend(sel, attn, apply, stream);
}

int imi_decode_layer(const imi_append_desc* app, const imi_async_desc* as, const imi_apply_desc* apply,
                     const imi_select_desc* sel, const imi_attn_desc* attn, void* stream) {
    if (app) {
        const int st = check_append(app);
        if (st != IMI_OK) return st;
    }
    if (as) {
        const int st = check_async(as);
        if (st != IMI_OK) return st;
    }
    {
        const int st = check_decode_attend(sel, attn, apply);
        if (st != IMI_OK) return st;
    }
    // Without an async assignment in this step nothing reads the appended
    // rows before the attention, so the select kernel does the append (one
    // launch and one programmatic hand-off fewer); the assignment reads the
    // batch slot that the append writes, so with it the append goes first.
    const bool fuse = app && !as && app->bg == sel->bg;
    if (app && !fuse) {
        cudaError_t e = imi::launch_append(*app, S(stream));
        if (e != cudaSuccess) return cuda_status(e, "imi_decode_layer(append)");
    }
    if (as) {
        cudaError_t e = imi::launch_async_assign(*as, S(stream));
        if (e != cudaSuccess) return cuda_status(e, "imi_decode_layer(async assignment)");
    }
    return launch_decode_attend(sel, attn, apply, stream, fuse ? app : nullptr);
}

int imi_merge_candidates(const imi_merge_desc* d, void* stream) {
    if (!d || !d->cand || !d->cell_offsets || !d->sel_cells || !d->sel_count ||
        !d->row_index || !d->row_count)
        return fail(IMI_ERR_INVALID, "imi_merge_candidates: null pointer");
    if (d->bg <= 0 || d->shards <= 0 || d->cap <= 0 || d->rank < 0 || d->rank >= d->shards || d->n_slots <= 0 ||
        d->nprobe <= 0 || d->nprobe > imi::select_max_slots() || d->page_size <= 0 || d->static_len < 0 || d->key_base < 0)
        return fail(IMI_ERR_INVALID, "imi_merge_candidates: bad sizes");
    if (d->cap > imi::select_max_slots() + 1)
        return fail(IMI_ERR_INVALID, "imi_merge_candidates: cap (nprobe + 1) too large");
    if (d->static_len + (int64_t)d->buffer_pages * d->page_size > d->exec_capacity)
        return fail(IMI_ERR_INVALID, "imi_merge_candidates: exec_capacity < static_len + buffer_pages*page_size");
    if (imi::merge_smem_bytes(*d) > 227 * 1024)
        return fail(IMI_ERR_INVALID, "imi_merge_candidates: shards * cap too large for one CTA's shared memory");
    return cuda_status(imi::launch_merge(*d, S(stream)), "imi_merge_candidates");
}

int imi_combine_partials(const imi_combine_desc* d, void* stream) {
    if (!d || !d->o_parts || !d->ml_parts || !d->out) return fail(IMI_ERR_INVALID, "imi_combine_partials: null pointer");
    if (d->shards <= 0 || d->bg <= 0 || d->G <= 0 || d->G > 8)
        return fail(IMI_ERR_INVALID, "imi_combine_partials: need shards, bg > 0 and 1 <= G <= 8");
    if (!aligned16(d->o_parts) || (d->part_stride % 4) != 0 || (reinterpret_cast<uintptr_t>(d->out) & 7u) != 0)
        return fail(IMI_ERR_INVALID, "imi_combine_partials: o_parts 16-byte, out 8-byte aligned");
    return cuda_status(imi::launch_combine_shards(*d, S(stream)), "imi_combine_partials");
}

int imi_peer_allgather(const imi_peer_gather_desc* d, void* stream) {
    if (!d || !d->src_peers || !d->flag_peers || !d->epoch || !d->ticket || !d->dst)
        return fail(IMI_ERR_INVALID, "imi_peer_allgather: null pointer");
    if (d->world <= 0 || d->world > 64 || d->rank < 0 || d->rank >= d->world || d->bytes <= 0 || d->bytes % 16 != 0 ||
        !aligned16(d->dst))
        return fail(IMI_ERR_INVALID, "imi_peer_allgather: need 0 <= rank < world <= 64, bytes a positive multiple of 16, "
                                     "dst 16-byte aligned");
    return cuda_status(imi::launch_peer_allgather(*d, S(stream)), "imi_peer_allgather");
}

int imi_decode_append(const imi_append_desc* d, void* stream) {
    const int st = check_append(d);
    if (st != IMI_OK) return st;
    return cuda_status(imi::launch_append(*d, S(stream)), "imi_decode_append");
}

int imi_async_assign(const imi_async_desc* d, void* stream) {
    const int st = check_async(d);
    if (st != IMI_OK) return st;
    return cuda_status(imi::launch_async_assign(*d, S(stream)), "imi_async_assign");
}

int imi_apply_updates(const imi_apply_desc* d, void* stream) {
    if (!d || !d->shadow || !d->live || !d->pending || !d->live_dirty)
        return fail(IMI_ERR_INVALID, "imi_apply_updates: null pointer");
    if (d->bg <= 0 || d->n_slots <= 0) return fail(IMI_ERR_INVALID, "imi_apply_updates: bad sizes");
    return cuda_status(imi::launch_apply(*d, S(stream)), "imi_apply_updates");
}

}  // extern "C"
