// imi_oracle.cpp -- CPU restatement of AdaptiveIMI's IMI KV-cache path.
//
// TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA path
// in adaptiveimi_b200/csrc.  Only tests/, __graft_entry__.smoke() and the CPU
// baseline / reference arm of bench.py may load it; the product never calls it.
//
// Parity is pinned: tests/test_oracle_pin.py checks every function here against
// the reference's own C++ (oracle/_ref, compiled in place from the reference
// sources by oracle/build_ref.py) and against the committed golden fixtures in
// tests/golden/ that were generated from that build.
//
// Every function names the reference file:line whose behaviour it restates.
// Paths are relative to the AdaptiveIMI project root.
//
// Written in C++ (not C) because the reference's k-means seeds are defined by
// libstdc++'s <random> (std::mt19937_64 / std::mt19937 with
// uniform_int_distribution / uniform_real_distribution); the same library is
// used here so the draws are the reference's draws.
//
// Build: g++ -O3 -march=x86-64-v3 -std=c++17 -ffp-contract=off -shared -fPIC (oracle/build_oracle.py)
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <limits>
#include <numeric>
#include <random>
#include <vector>

namespace {

inline float bf16_to_f32(uint16_t h) {
    uint32_t u = static_cast<uint32_t>(h) << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

// Squared L2 distance with the reference's lane order:
// kmeans_core.cpp:22-44 (euclidean_distance_avx2): eight fp32 lanes, lane l
// accumulates fma(d, d, acc) over dims l, l+8, ...; the lanes are then added
// left to right; any tail (dim % 8) is added after with a separate multiply.
inline float dist_l2_lanes8(const float* a, const float* b, int dim) {
    float lane[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int i = 0;
    for (; i + 7 < dim; i += 8) {
        for (int l = 0; l < 8; ++l) {
            float d = a[i + l] - b[i + l];
            lane[l] = std::fma(d, d, lane[l]);
        }
    }
    float total = lane[0] + lane[1] + lane[2] + lane[3] + lane[4] + lane[5] + lane[6] + lane[7];
    for (; i < dim; ++i) {
        float d = a[i] - b[i];
        total += d * d;
    }
    return total;
}

// k-means++ seeding: kmeans_core.cpp:138-186.
void kmeanspp_init(const float* data, int n, int dim, int k, uint64_t seed, float* cent) {
    std::vector<float> min_d(n, std::numeric_limits<float>::max());
    std::mt19937_64 rng(seed);
    std::uniform_int_distribution<int32_t> pick(0, n - 1);
    int first = pick(rng);
    std::memcpy(cent, data + static_cast<size_t>(first) * dim, sizeof(float) * dim);
    for (int c = 1; c < k; ++c) {
        const float* prev = cent + static_cast<size_t>(c - 1) * dim;
        for (int i = 0; i < n; ++i) {
            float d = dist_l2_lanes8(data + static_cast<size_t>(i) * dim, prev, dim);
            if (d < min_d[i]) min_d[i] = d;
        }
        double total = 0.0;
        for (int i = 0; i < n; ++i) total += min_d[i];
        std::uniform_real_distribution<double> u(0.0, total);
        double target = u(rng);
        double run = 0.0;
        int sel = 0;
        for (int i = 0; i < n; ++i) {
            run += min_d[i];
            if (run >= target) {
                sel = i;
                break;
            }
        }
        std::memcpy(cent + static_cast<size_t>(c) * dim, data + static_cast<size_t>(sel) * dim, sizeof(float) * dim);
    }
}

// Lloyd iterations with one worker thread: kmeans_core.cpp:190-314.
// E-step first-min argmin (:218-241); early stop (:243-262); M-step sums in
// sample order (:268-296 with one thread); mean = sum * (1/size) (:303-307);
// empty cell reseeded from mt19937(iter + 12345) (:299-311).
// Returns the number of iterations entered.
int lloyd(const float* data, int n, int dim, int k, float* cent, int32_t* labels, int max_iters, float tol,
          int min_iter, float rel_tol, float* inertia_out) {
    std::vector<float> sums(static_cast<size_t>(k) * dim);
    std::vector<int32_t> sizes(k);
    float prev = std::numeric_limits<float>::max();
    float inertia = 0.0f;
    int iters = 0;
    for (int it = 0; it < max_iters; ++it) {
        ++iters;
        inertia = 0.0f;
        for (int i = 0; i < n; ++i) {
            float best = std::numeric_limits<float>::max();
            int32_t bi = 0;
            for (int c = 0; c < k; ++c) {
                float d = dist_l2_lanes8(data + static_cast<size_t>(i) * dim, cent + static_cast<size_t>(c) * dim, dim);
                if (d < best) {
                    best = d;
                    bi = c;
                }
            }
            labels[i] = bi;
            inertia += best;
        }
        float change = std::fabs(prev - inertia);
        float rel = prev > 0 ? change / prev : 0.0f;
        if (iters >= std::max(1, min_iter) && (rel <= std::max(0.0f, rel_tol) || change <= std::max(0.0f, tol))) break;
        prev = inertia;
        std::fill(sums.begin(), sums.end(), 0.0f);
        std::fill(sizes.begin(), sizes.end(), 0);
        for (int i = 0; i < n; ++i) {
            int c = labels[i];
            sizes[c]++;
            for (int d = 0; d < dim; ++d) sums[static_cast<size_t>(c) * dim + d] += data[static_cast<size_t>(i) * dim + d];
        }
        std::mt19937 rng(it + 12345);
        std::uniform_int_distribution<int32_t> pick(0, n - 1);
        for (int c = 0; c < k; ++c) {
            if (sizes[c] > 0) {
                float inv = 1.0f / static_cast<float>(sizes[c]);
                for (int d = 0; d < dim; ++d) cent[static_cast<size_t>(c) * dim + d] = sums[static_cast<size_t>(c) * dim + d] * inv;
            } else {
                int s = pick(rng);
                std::memcpy(cent + static_cast<size_t>(c) * dim, data + static_cast<size_t>(s) * dim, sizeof(float) * dim);
            }
        }
    }
    if (inertia_out) *inertia_out = inertia;
    return iters;
}

}  // namespace

extern "C" {

int oracle_abi_version() { return 1; }

// One (head, subspace) k-means task: kmeans_core.cpp:351-382
// (run_imi_single_phase_from_subvec).  data: [n, dim] fp32.
int oracle_kmeans(const float* data, int n, int dim, int k, uint64_t seed, int max_iters, float tol, int min_iter,
                  float rel_tol, int32_t* labels, float* centroids, float* inertia) {
    if (n <= 0 || k <= 0) return -1;
    kmeanspp_init(data, n, dim, k, seed, centroids);
    return lloyd(data, n, dim, k, centroids, labels, max_iters, tol, min_iter, rel_tol, inertia);
}

// k-means++ seeding only (kmeans_core.cpp:138-186), for kernel-level tests.
int oracle_kmeanspp(const float* data, int n, int dim, int k, uint64_t seed, float* centroids) {
    if (n <= 0 || k <= 0) return -1;
    kmeanspp_init(data, n, dim, k, seed, centroids);
    return 0;
}

// Whole-head IMI build: k-means over `parts` subspaces (parts = 2 or 4; 0 = IVF
// on the full vector), then the compact + CSR reorganize.
//   kmeans_core.cpp:384-501 (IMI-2), :503-595 (IVF), :598-772 (IMI-4), seeds
//   42, 43, 44, 45 per subspace (:459,:469,:704-734);
//   reorganize_core.cpp:18-85 / :87-176 / :178-231 (compact ids in ascending
//   Cartesian order, counts, exclusive offsets, merged centroid = concatenation
//   of subspace centroids) and :234-311 (stable counting-sort permutation, rows
//   copied in list order).
// keys/values: [n, dim] bf16 bits.  ks: per-subspace k (ks[0] for IVF).
// Outputs: sub_labels [parts_or_1, n]; sub_centroids packed per subspace
// (subspace s at offset sum_{t<s} ks[t]*sub_dim); final_labels [n] (compact);
// offsets [n_active+1] (caller provides n+1 capacity... at most prod(ks)+1);
// merged [n_active, dim]; list_keys/list_values [n, dim] bf16 bits.
// Returns n_active (>= 1) or -1.
int oracle_build_head(const uint16_t* keys, const uint16_t* values, int n, int dim, int parts, const int* ks,
                      int max_iters, float tol, int min_iter, float rel_tol, int32_t* sub_labels, float* sub_centroids,
                      int32_t* final_labels, int32_t* offsets, float* merged, uint16_t* list_keys,
                      uint16_t* list_values, int32_t* iters_out) {
    if (n <= 0) return -1;
    const int S = parts == 0 ? 1 : parts;
    const int sub = dim / S;
    std::vector<float> full(static_cast<size_t>(n) * dim);
    for (size_t i = 0; i < full.size(); ++i) full[i] = bf16_to_f32(keys[i]);
    std::vector<float> subv(static_cast<size_t>(n) * sub);
    size_t coff = 0;
    for (int s = 0; s < S; ++s) {
        for (int i = 0; i < n; ++i)
            std::memcpy(&subv[static_cast<size_t>(i) * sub], &full[static_cast<size_t>(i) * dim + s * sub], sizeof(float) * sub);
        int it = oracle_kmeans(subv.data(), n, sub, ks[s], 42 + s, max_iters, tol, min_iter, rel_tol,
                               sub_labels + static_cast<size_t>(s) * n, sub_centroids + coff, nullptr);
        if (iters_out) iters_out[s] = it;
        coff += static_cast<size_t>(ks[s]) * sub;
    }
    // Cartesian id in mixed radix, first subspace most significant.
    int64_t total = 1;
    for (int s = 0; s < S; ++s) total *= ks[s];
    std::vector<int64_t> comb(n);
    for (int i = 0; i < n; ++i) {
        int64_t id = 0;
        for (int s = 0; s < S; ++s) id = id * ks[s] + sub_labels[static_cast<size_t>(s) * n + i];
        comb[i] = id;
    }
    std::vector<int32_t> g2c(static_cast<size_t>(total), -1);
    for (int i = 0; i < n; ++i) g2c[comb[i]] = 1;
    int n_active = 0;
    for (int64_t g = 0; g < total; ++g)
        if (g2c[g] == 1) g2c[g] = n_active++; else g2c[g] = -1;
    std::vector<int32_t> counts(n_active, 0);
    for (int i = 0; i < n; ++i) {
        final_labels[i] = g2c[comb[i]];
        counts[final_labels[i]]++;
    }
    offsets[0] = 0;
    for (int c = 0; c < n_active; ++c) offsets[c + 1] = offsets[c] + counts[c];
    // merged centroids
    for (int64_t g = 0; g < total; ++g) {
        int c = g2c[g];
        if (c < 0) continue;
        int64_t rem = g;
        std::vector<int> digit(S);
        for (int s = S - 1; s >= 0; --s) {
            digit[s] = static_cast<int>(rem % ks[s]);
            rem /= ks[s];
        }
        size_t so = 0;
        for (int s = 0; s < S; ++s) {
            std::memcpy(merged + static_cast<size_t>(c) * dim + s * sub, sub_centroids + so + static_cast<size_t>(digit[s]) * sub,
                        sizeof(float) * sub);
            so += static_cast<size_t>(ks[s]) * sub;
        }
    }
    // stable counting sort of rows
    std::vector<int32_t> pos(offsets, offsets + n_active);
    for (int i = 0; i < n; ++i) {
        int p = pos[final_labels[i]]++;
        std::memcpy(list_keys + static_cast<size_t>(p) * dim, keys + static_cast<size_t>(i) * dim, 2 * dim);
        std::memcpy(list_values + static_cast<size_t>(p) * dim, values + static_cast<size_t>(i) * dim, 2 * dim);
    }
    return n_active;
}

// Cell scores for one KV group: compute_impl.cu:62-103
// (fused_query_group_similarity_kernel): q_sum[d] = sum_g float(q[g,d]) in g
// order, then sim[c] = fma chain over d = 0..dim-1 (nvcc contracts
// `sim += q*c` into fma).  Masked slots are set to -inf afterwards
// (retrieval.py:357).
void oracle_scores(const uint16_t* q, int G, int dim, const float* cent, const uint8_t* mask, int n_slots,
                   float* out) {
    std::vector<float> qs(dim);
    for (int d = 0; d < dim; ++d) {
        float acc = 0.0f;
        for (int g = 0; g < G; ++g) acc += bf16_to_f32(q[static_cast<size_t>(g) * dim + d]);
        qs[d] = acc;
    }
    for (int c = 0; c < n_slots; ++c) {
        float s = 0.0f;
        for (int d = 0; d < dim; ++d) s = std::fma(qs[d], cent[static_cast<size_t>(c) * dim + d], s);
        out[c] = (mask && mask[c]) ? -std::numeric_limits<float>::infinity() : s;
    }
}

// Cell selection for one KV group:
//   retrieval.py:295-303 (_select_clusters): top-nprobe by score (ties: lower
//   slot first), keep = size > 0 and exclusive size cumsum < max_tokens;
//   wave_buffer_cpu_hotcold.cpp:303-371 (BufferManager::batch_access): walk the
//   kept cells in order, skip empty ones, stop before the cell whose pages
//   ceil(size/page) push the running page count above buffer_pages.
// Writes the surviving cells in score order to out_cells; returns their count.
// If pre_trunc is non-null it receives the nprobe-long list after the budget
// rule, with padding_id for dropped entries (what the reference passes on).
int oracle_select(const float* scores, const int32_t* sizes, int n_slots, int nprobe, int max_tokens,
                  int buffer_pages, int page_size, int padding_id, int32_t* out_cells, int32_t* pre_trunc) {
    std::vector<int32_t> idx(n_slots);
    std::iota(idx.begin(), idx.end(), 0);
    std::stable_sort(idx.begin(), idx.end(), [&](int32_t a, int32_t b) { return scores[a] > scores[b]; });
    const int m = std::min(nprobe, n_slots);
    int32_t cum = 0;
    std::vector<int32_t> kept(m);
    for (int r = 0; r < m; ++r) {
        int32_t c = idx[r];
        int32_t sz = sizes[c];
        cum += sz;
        bool keep = sz > 0 && (cum - sz) < max_tokens;
        kept[r] = keep ? c : padding_id;
        if (pre_trunc) pre_trunc[r] = kept[r];
    }
    int out = 0;
    int pages = 0;
    for (int r = 0; r < m; ++r) {
        int32_t c = kept[r];
        int32_t sz = (c >= 0 && c < n_slots) ? sizes[c] : 0;
        if (sz <= 0) continue;
        pages += (sz + page_size - 1) / page_size;
        if (pages > buffer_pages) break;
        out_cells[out++] = c;
    }
    return out;
}

// Softmax attention of G query heads over `rows` K/V rows (bf16 bits), in
// double: the semantics of weighted_flash_decoding as called at
// retrieval.py:439-447 (softmax(scale * q.K^T) V per KV group).  out: [G, dim].
void oracle_attention(const uint16_t* q, int G, int dim, const uint16_t* k_rows, const uint16_t* v_rows, int rows,
                      double scale, double* out) {
    std::vector<double> s(rows);
    for (int g = 0; g < G; ++g) {
        double mx = -INFINITY;
        for (int r = 0; r < rows; ++r) {
            double acc = 0;
            for (int d = 0; d < dim; ++d)
                acc += static_cast<double>(bf16_to_f32(q[g * dim + d])) * bf16_to_f32(k_rows[static_cast<size_t>(r) * dim + d]);
            s[r] = acc * scale;
            mx = std::max(mx, s[r]);
        }
        double l = 0;
        for (int r = 0; r < rows; ++r) {
            s[r] = std::exp(s[r] - mx);
            l += s[r];
        }
        for (int d = 0; d < dim; ++d) {
            double acc = 0;
            for (int r = 0; r < rows; ++r) acc += s[r] * bf16_to_f32(v_rows[static_cast<size_t>(r) * dim + d]);
            out[g * dim + d] = rows > 0 ? acc / l : 0.0;
        }
    }
}

// One batched async centroid update for one KV group: async_update.py:122-143.
// keys: [B, dim] bf16 bits; shadow: [n_slots, dim] fp32 (updated in place);
// counts / delta_counts: [n_slots] int32; delta_sums: [n_slots, dim] fp32.
// Inner products use a d-ordered fma chain (the reference uses torch.bmm, whose
// accumulation order is cuBLAS's; see the near-tie note in the tests).  Ties go
// to the lowest slot (torch.argmax returns the first maximum).  Sums are added
// in token order.  cell_ids: [B] output.
void oracle_async_update(const uint16_t* keys, int B, int dim, float* shadow, int n_slots, int32_t* counts,
                         int32_t* delta_counts, float* delta_sums, int threshold, int32_t* cell_ids) {
    std::vector<float> kf(static_cast<size_t>(B) * dim);
    for (size_t i = 0; i < kf.size(); ++i) kf[i] = bf16_to_f32(keys[i]);
    for (int b = 0; b < B; ++b) {
        float best = -std::numeric_limits<float>::infinity();
        int bi = 0;
        for (int c = 0; c < n_slots; ++c) {
            float s = 0.0f;
            for (int d = 0; d < dim; ++d) s = std::fma(kf[b * dim + d], shadow[static_cast<size_t>(c) * dim + d], s);
            if (s > best) {
                best = s;
                bi = c;
            }
        }
        cell_ids[b] = bi;
    }
    for (int b = 0; b < B; ++b) {
        int c = cell_ids[b];
        delta_counts[c] += 1;
        for (int d = 0; d < dim; ++d) delta_sums[static_cast<size_t>(c) * dim + d] += kf[b * dim + d];
    }
    for (int c = 0; c < n_slots; ++c) {
        if (delta_counts[c] < threshold) continue;
        int32_t nc = counts[c] + delta_counts[c];
        float denom = static_cast<float>(std::max(nc, 1));
        float cnt = static_cast<float>(counts[c]);
        for (int d = 0; d < dim; ++d) {
            size_t o = static_cast<size_t>(c) * dim + d;
            shadow[o] = (shadow[o] * cnt + delta_sums[o]) / denom;
            delta_sums[o] = 0.0f;
        }
        counts[c] = nc;
        delta_counts[c] = 0;
    }
}

}  // extern "C"
