/*
 * imi_b200.h -- C ABI of the B200 (sm_100a) implementation of AdaptiveIMI's
 * inverted-multi-index (IMI) KV-cache path.
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t
 * (passed as void*), launches asynchronously on that stream, allocates no
 * memory (scratch is passed in by the caller), and returns 0 on success or a
 * nonzero status; imi_last_error() then describes the failure (thread-local).
 *
 * Tensor layouts (all row-major, contiguous unless a stride is given):
 *   bf16 values are passed as their 16-bit patterns.
 *   bg = batch * kv_heads ("KV groups"), G = query heads per KV group,
 *   D = head dim (128), S = subspace parts (2, 4; 0 means IVF with one part),
 *   n_slots = cell slots per group (padded, = reference n_centroids).
 *
 * Reference interfaces replaced (paths relative to the AdaptiveIMI project):
 *   imi_build_index        imi::kmeans_execute{,_4,_ivf} (kmeans_core.cpp:822-1174)
 *                          + imi::reorganize_from_kmeans{,_4,_ivf}
 *                          (reorganize_core.cpp:313-569) + metadata padding
 *                          (pipeline_bindings.cpp:206-276, indexing.py:108-174),
 *                          i.e. the LayerPipeline merge path
 *                          (layer_pipeline.cpp:1077-1401)
 *   imi_query_group_similarities
 *                          gpu_cluster_manager_cpp.fused_query_group_similarities
 *                          (compute_wrappers.cpp:39-104, compute_impl.cu:62-103)
 *   imi_select_cells       AdaptiveIMIRetrievalMixin._select_clusters
 *                          (retrieval.py:295-303) + AdpIMI_Index.batch_access
 *                          page truncation (wave_buffer_cpu_hotcold.cpp:303-371,
 *                          897-929) + the execution-buffer layout of
 *                          Copy.gather_copy_and_concat (gather_copy.cu:100-213)
 *                          + the delta-row match of _append_delta_to_execution
 *                          (async_update.py:20-76)
 *   imi_sparse_attention   the gather of gather_copy_and_concat fused with
 *                          weighted_flash_decoding (retrieval.py:439-447)
 *   imi_decode_attend      the whole decode attention of one layer,
 *                          AdaptiveIMIRetrievalMixin.sparse_attention
 *                          (retrieval.py:320-602): apply + select + attention
 *   imi_decode_append      decode_update_kv_cache (runtime.py:378-392) and the
 *                          async-update batch buffer (async_update.py:112-117)
 *   imi_async_assign       _schedule_async_update batch step (async_update.py:118-161)
 *   imi_apply_updates      _apply_async_centroid_updates (async_update.py:7-19)
 */
#ifndef IMI_B200_H_
#define IMI_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define IMI_ABI_VERSION 2

#if defined(__GNUC__)
#define IMI_API __attribute__((visibility("default")))
#else
#define IMI_API
#endif

#define IMI_OK 0
#define IMI_ERR_INVALID 1
#define IMI_ERR_CUDA 2

/* Row-list entries written by imi_select_cells: (source << 30) | row, where
 * source 0 = IMI list row, 1 = steady-zone row, 2 = delta-ring row (the value is
 * then negative as int32; -1 is never a valid entry).  The list holds the
 * steady-zone rows, then the selected cells' rows (cells in slot order), then
 * the matching delta rows. */
#define IMI_ROW_SOURCE_SHIFT 30

/* Size of the library-owned scratch array used by imi_sparse_attention_noalloc. */
#define IMI_NOALLOC_SCRATCH_BYTES (1u << 20)

typedef struct imi_build_desc {
    int32_t heads, n_tokens, dim, parts;   /* parts: 0 (IVF), 2 or 4 */
    int32_t ks[4];                         /* k per subspace (ks[0] for IVF) */
    const uint16_t* keys;                  /* bf16, element (h,i,d) at keys[h*head_stride + i*token_stride + d] */
    const uint16_t* values;
    int64_t head_stride, token_stride;     /* in elements; 16-byte aligned */
    int32_t max_iters, early_stop_min_iter;
    float tol, early_stop_rel_tol;
    uint16_t* list_keys;                   /* [heads, list_rows, dim] out: rows in cell (CSR) order */
    uint16_t* list_values;
    int64_t list_rows;                     /* >= n_tokens */
    int32_t n_slots, kmax;                 /* padded slots per head; sub-centroid stride (>= max k) */
    int32_t* cell_sizes;                   /* [heads, n_slots] */
    int32_t* cell_offsets;                 /* [heads, n_slots + 1] */
    uint8_t* cell_mask;                    /* [heads, n_slots] 1 = empty / padding */
    int32_t* cell_code;                    /* [heads, n_slots] packed subspace digits, -1 = padding */
    float* centroids;                      /* [heads, n_slots, dim] merged centroids (zeros for padding) */
    float* sub_centroids;                  /* [heads, S, kmax, dim/S] */
    int32_t* sub_labels;                   /* [heads, S, n_tokens] or NULL (kept in the workspace) */
    int32_t* n_active;                     /* [heads] active cells */
    int32_t* iters_run;                    /* [heads, S] Lloyd iterations entered, or NULL */
    void* workspace;
    size_t workspace_bytes;
    int32_t* status;                       /* [1] or NULL: bit 0 is set when a wait of the tensor-core
                                              E-step gave up (the index is then not valid; the labels
                                              that CTA owned are left at 0 so that later kernels stay
                                              in bounds) */
    unsigned long long* phase_ns;          /* [3] or NULL: device timestamps (ns, globaltimer) taken on
                                              the stream when k-means starts, when it ends and when
                                              the reorganize (CSR lists, padded metadata, list rows)
                                              ends: the per-stage times of PipelineStats */
    void* ready_event;                     /* cudaEvent_t or NULL: recorded where keys / values are
                                              produced; the build's stream waits for it after staging
                                              its seeded draws and before the first kernel, so the
                                              build can run on a side stream next to the producer */
} imi_build_desc;

typedef struct imi_select_desc {
    int32_t bg, G, dim, n_slots, parts, kmax;
    int32_t ks[4];
    const uint16_t* q;                     /* [bg, G, dim] */
    const float* sub_centroids;            /* [bg, S, kmax, dim/S] */
    const int32_t* cell_code;              /* [bg, n_slots] */
    const int32_t* cell_sizes;             /* [bg, n_slots] */
    const int32_t* cell_offsets;           /* [bg, n_slots + 1] */
    const uint8_t* cell_mask;              /* [bg, n_slots] */
    const float* centroids;                /* [bg, n_slots, dim] live merged centroids */
    const uint8_t* cell_dirty;             /* [bg, n_slots] or NULL: 1 = live centroid was updated */
    int32_t nprobe, max_tokens, buffer_pages, page_size, padding_id;
    int32_t static_len;
    const int32_t* delta_cell_ids;         /* [bg, delta_capacity] or NULL */
    const int32_t* delta_count;            /* [bg] or NULL */
    int32_t delta_capacity;
    int32_t exec_capacity;                 /* row-list capacity (>= static_len + buffer_pages*page_size) */
    int32_t* sel_cells;                    /* [bg, nprobe] out: selected cells, ascending slot order */
    int32_t* sel_count;                    /* [bg] out */
    int32_t* kept_count;                   /* [bg] out or NULL: cells kept before page truncation */
    int32_t* row_index;                    /* [bg, exec_capacity] out */
    int32_t* row_count;                    /* [bg] out */
    float* scores_out;                     /* [bg, n_slots] out or NULL */
    unsigned long long* phase_ns;          /* [bg, 8] out or NULL: device timestamps (ns) of the
                                              selection's phases, a profiling aid */
    int32_t slot_bound;                    /* 0, or a bound on the occupied slots: every slot at or
                                              above it is masked (padding) in every group, e.g. the
                                              largest n_active of the build; the kernel skips them */
    int32_t key_base;                      /* 0, or this shard's global cell-id offset: ties between
                                              equal scores go to the lower key_base + slot */
    unsigned long long* cand_out;          /* [bg, 2 * (nprobe + 1) + 1] out or NULL: this shard's
                                              candidates for imi_merge_candidates -- ranking keys
                                              (ordered score bits, then ~(key_base + slot)) of the
                                              selected cells in slot order, then the stop marker (the
                                              highest-ranked cell left out, if any); their sizes from
                                              offset nprobe + 1; the entry count last */
} imi_select_desc;

typedef struct imi_attn_desc {
    int32_t bg, G, splits, exec_capacity;  /* dim is 128; G <= 8, splits <= 4096, splits * G <= 16384 */
    float scale;
    const uint16_t* q;                     /* [bg, G, 128] */
    const int32_t* row_index;              /* [bg, exec_capacity] */
    const int32_t* row_count;              /* [bg] */
    const void* list_keys;                 /* [bg, list_rows, 128] */
    const void* list_values;
    int64_t list_rows;
    const void* static_keys;               /* [bg, static_rows, 128] */
    const void* static_values;
    int64_t static_rows;
    const void* delta_keys;                /* [bg, delta_rows, 128] or NULL */
    const void* delta_values;
    int64_t delta_rows;
    float* part_o;                         /* scratch [bg, splits, G, 128], 16-byte aligned */
    float* part_ml;                        /* scratch [bg, splits, G, 2], 8-byte aligned */
    void* out;                             /* [bg, G, 128] bf16 out, 8-byte aligned */
    int32_t* counters;                     /* scratch [bg], zero before the first call, or NULL:
                                              with it the last CTA of a group merges the
                                              splits (and re-zeroes its counter); without it a
                                              separate merge kernel runs */
    int32_t* status;                       /* [1] or NULL: reserved.  The attention kernels have no
                                              spin-waits (row copies are cp.async groups, the split
                                              merge is a ticket), so no bit is set; callers may pass
                                              NULL */
    float* o_part;                         /* [bg, G, 128] out or NULL: unnormalised output (sequence
                                              sharding); needs counters */
    float* ml_part;                        /* [bg, G, 2] out or NULL: (max in log2 units, sum) */
} imi_attn_desc;

/* Sequence sharding: the global selection over every shard's candidates.
 * Each shard ran imi_select_cells under the global rules with key_base = its
 * global cell-id offset and row_index = NULL; its candidates are its selected
 * cells (slot order) followed by its stop marker (next_key).  Every shard runs
 * this merge on the same all-gathered candidates, so every shard finds the same
 * boundary; it then writes its own selected cells and row list. */
typedef struct imi_merge_desc {
    int32_t bg, shards, cap;               /* cap = nprobe + 1 (the select's candidate slots) */
    int32_t rank;                          /* this shard */
    int32_t key_base;                      /* this shard's global cell-id offset */
    const unsigned long long* cand;        /* [shards, bg, 2 * cap + 1]: every shard's cand_out */
    const int32_t* cell_offsets;           /* this shard's [bg, n_slots + 1] */
    int32_t n_slots;                       /* this shard's slots */
    int32_t nprobe, max_tokens, buffer_pages, page_size;  /* the global rules */
    int32_t static_len;                    /* steady-zone rows this shard attends (0 on all but one) */
    int32_t exec_capacity;
    int32_t* sel_cells;                    /* [bg, nprobe] out: this shard's selected slots, ascending */
    int32_t* sel_count;                    /* [bg] out */
    int32_t* row_index;                    /* [bg, exec_capacity] out */
    int32_t* row_count;                    /* [bg] out */
} imi_merge_desc;

/* Sequence sharding: combine the shards' unnormalised attention partials
 * (imi_attn_desc o_part / ml_part) by log-sum-exp into the bf16 output. */
typedef struct imi_combine_desc {
    int32_t shards, bg, G;
    int64_t part_stride;                   /* floats from one shard's partials to the next */
    const float* o_parts;                  /* shard s: [bg, G, 128] at o_parts + s * part_stride */
    const float* ml_parts;                 /* shard s: [bg, G, 2] at ml_parts + s * part_stride:
                                              (max in log2 units, sum) */
    void* out;                             /* [bg, G, 128] bf16 */
} imi_combine_desc;

/* Sequence sharding: all-gather of one block per rank over NVLink peer memory
 * (no counterpart in the reference).  src_peers[r] is rank r's source block
 * (bytes long, 16-byte aligned) as mapped on this GPU; flag_peers[r] is rank
 * r's array of `world` flag words as mapped on this GPU (zero before the
 * first call); epoch and ticket are this rank's own counters (zero before the
 * first call, advanced by the kernel).  Both arrays live in device memory.
 * dst receives [world][bytes].  A peer that does not arrive within about a
 * second sets bit 0 of *status. */
typedef struct imi_peer_gather_desc {
    int32_t world, rank;
    int64_t bytes;                         /* per rank, a multiple of 16 */
    const void* const* src_peers;          /* [world] device array of peer pointers */
    uint32_t* const* flag_peers;           /* [world] device array of peer pointers */
    uint32_t* epoch;                       /* [1] this rank's exchange counter */
    uint32_t* ticket;                      /* [1] scratch, zero between calls */
    void* dst;                             /* [world, bytes] */
    int32_t* status;                       /* [1] or NULL */
} imi_peer_gather_desc;

typedef struct imi_append_desc {
    int32_t bg, dim;
    const void* new_keys;                  /* group h at new_keys + h*src_head_stride elements */
    const void* new_values;
    int64_t src_head_stride;
    void* zone_keys;                       /* [bg, zone_rows, dim] */
    void* zone_values;
    int64_t zone_rows;
    int32_t pos;
    void* batch_keys;                      /* [bg, batch_cap, dim] or NULL */
    void* batch_values;
    int32_t batch_cap, batch_slot;
} imi_append_desc;

typedef struct imi_async_desc {
    int32_t bg, dim, n_slots, parts, kmax, batch, batch_cap, threshold, ring_cap;
    int32_t ks[4];
    const uint16_t* batch_keys;            /* [bg, batch_cap, dim] */
    const uint16_t* batch_values;
    const float* sub_centroids;            /* [bg, S, kmax, dim/S] */
    const int32_t* cell_code;              /* [bg, n_slots] */
    float* shadow;                         /* [bg, n_slots, dim] */
    uint8_t* shadow_dirty;                 /* [bg, n_slots] */
    uint8_t* pending;                      /* [bg, n_slots] */
    int32_t* counts;                       /* [bg, n_slots] */
    int32_t* delta_counts;                 /* [bg, n_slots] */
    float* delta_sums;                     /* [bg, n_slots, dim] */
    uint16_t* ring_keys;                   /* [bg, ring_cap, dim] */
    uint16_t* ring_values;
    int32_t* ring_cell_ids;                /* [bg, ring_cap] */
    int32_t* ring_write_pos;               /* [bg] */
    int32_t* ring_count;                   /* [bg] */
    int32_t* ids_out;                      /* [bg, batch] or NULL */
    unsigned long long* part_best;         /* scratch [bg, part_chunks, batch] */
    int32_t part_chunks;                   /* = ceil(n_slots / 512) */
    int32_t ring_store;                    /* 0: the ring's rows and cell ids are left as they are and
                                              only its write position and count advance -- what the
                                              reference does: its `ring[g, pos].copy_(x)` with a tensor
                                              index `pos` (async_update.py:151-157) writes into a
                                              temporary, so its ring keeps zero rows and padding ids;
                                              1: the batch's keys, values and cells are stored */
} imi_async_desc;

typedef struct imi_apply_desc {
    int32_t bg, n_slots, dim;
    const float* shadow;
    float* live;
    uint8_t* pending;
    uint8_t* live_dirty;
} imi_apply_desc;

IMI_API int imi_abi_version(void);
IMI_API const char* imi_last_error(void);

IMI_API size_t imi_build_workspace_size(int32_t heads, int32_t n_tokens, int32_t dim, int32_t parts, const int32_t* ks);
IMI_API int imi_build_index(const imi_build_desc* desc, void* stream);

IMI_API int imi_query_group_similarities(const uint16_t* q, const float* centroids, float* out, int32_t kv_heads,
                                 int32_t groups, int32_t n_clusters, int32_t dim, int64_t out_stride, void* stream);
IMI_API int imi_select_cells(const imi_select_desc* desc, void* stream);
IMI_API int imi_sparse_attention(const imi_attn_desc* desc, void* stream);
/* imi_sparse_attention without caller-provided scratch.  This entry point has
 * no counterpart in the reference.  It exists for callers that cannot allocate
 * device memory at all (code running inside another allocator, a host callback,
 * or a runtime that forbids cudaMalloc after start-up) and therefore cannot pass
 * part_o / part_ml / counters: those fields of the descriptor are ignored and a
 * fixed array owned by the library (IMI_NOALLOC_SCRATCH_BYTES, 1 MiB per GPU
 * that loads the library, held until the process exits) is used instead.
 * Limit: bg * splits * G * 520 bytes plus alignment must fit in that array;
 * larger requests fail with IMI_ERR_INVALID and a message.  The first call on
 * a device looks the array's address up (cudaGetSymbolAddress); make that first
 * call before any stream capture.  All calls share the one array, so calls that
 * can overlap on the GPU (other streams, other host threads) race: serialise
 * them.  It allocates nothing (no cudaMalloc/cudaFree). */
IMI_API int imi_sparse_attention_noalloc(const imi_attn_desc* desc, void* stream);
/* apply (optional, NULL to skip) + select + attention in one call: the per-layer
 * decode attention of the cache (retrieval.py:320-602).  sel and attn must name
 * the same q, row_index, row_count and exec_capacity. */
IMI_API int imi_decode_attend(const imi_select_desc* sel, const imi_attn_desc* attn, const imi_apply_desc* apply,
                              void* stream);
/* One decode layer in one call: append (NULL to skip), the batched cell
 * assignment (NULL to skip; runs after the append), apply (NULL to skip),
 * select and attention -- the order of decode_update_kv_cache followed by
 * attn_func (runtime.py:378-392, async_update.py:112-161, retrieval.py:320-602).
 * Every descriptor is validated before the first launch. */
IMI_API int imi_decode_layer(const imi_append_desc* append, const imi_async_desc* async_assign,
                             const imi_apply_desc* apply, const imi_select_desc* sel, const imi_attn_desc* attn,
                             void* stream);
IMI_API int imi_decode_append(const imi_append_desc* desc, void* stream);
/* Sequence sharding (no counterpart in the reference: its cache is one GPU):
 * the global candidate merge and the partial combine. */
IMI_API int imi_merge_candidates(const imi_merge_desc* desc, void* stream);
IMI_API int imi_combine_partials(const imi_combine_desc* desc, void* stream);
IMI_API int imi_peer_allgather(const imi_peer_gather_desc* desc, void* stream);
IMI_API int imi_async_assign(const imi_async_desc* desc, void* stream);
IMI_API int imi_apply_updates(const imi_apply_desc* desc, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* IMI_B200_H_ */
