// Test-only shim around the reference's own CPU index-build code.
//
// This file is test infrastructure: it is compiled (by oracle/build_ref.py)
// together with the reference sources `library/AdaptiveIMI/cpp_extensions/src/
// kmeans_core.cpp` and `reorganize_core.cpp`, read in place from the reference
// checkout, into `oracle/_ref/imi_ref*.so`.  Only tests, the smoke check and the
// bench's CPU-baseline / reference arm load it.  It never ships in the product.
//
// It exposes the two public entry points the reference's LayerPipeline calls:
//   imi::kmeans_execute{,_4,_ivf}   (kmeans_core.cpp:822-1174)
//   imi::reorganize_from_kmeans{,_4,_ivf} (reorganize_core.cpp:313-569)
// with a deterministic runtime config (worker threads chosen by the caller; the
// reference's M-step sums depend on the thread count, kmeans_core.cpp:268-296).
#include <torch/extension.h>
#include <vector>
#include <memory>
#include "layer_pipeline.hpp"

namespace py = pybind11;

namespace {

imi::LayerPipelineRuntimeConfig make_cfg(int max_iters, double tol, int min_iter, double rel_tol) {
    imi::LayerPipelineRuntimeConfig cfg;
    cfg.worker_threads = 1;
    cfg.enable_omp_nested = false;
    cfg.min_threads_per_phase = 1;
    cfg.kmeans_max_iters = max_iters;
    cfg.kmeans_tol = static_cast<float>(tol);
    cfg.kmeans_early_stop_min_iter = min_iter;
    cfg.kmeans_early_stop_rel_tol = static_cast<float>(rel_tol);
    return cfg;
}

torch::Tensor vec2d_i32(const std::vector<std::vector<int32_t>>& v, int64_t cols) {
    auto t = torch::zeros({static_cast<int64_t>(v.size()), cols}, torch::kInt32);
    for (size_t h = 0; h < v.size(); ++h) {
        std::memcpy(t[h].data_ptr<int32_t>(), v[h].data(), sizeof(int32_t) * std::min<size_t>(cols, v[h].size()));
    }
    return t;
}

torch::Tensor vec2d_f32(const std::vector<std::vector<float>>& v, int64_t rows, int64_t cols) {
    auto t = torch::zeros({static_cast<int64_t>(v.size()), rows, cols}, torch::kFloat32);
    for (size_t h = 0; h < v.size(); ++h) {
        std::memcpy(t[h].data_ptr<float>(), v[h].data(), sizeof(float) * std::min<size_t>(rows * cols, v[h].size()));
    }
    return t;
}

// keys: [kv_heads, n, dim] bfloat16 (CPU, contiguous)
py::dict kmeans(torch::Tensor keys, int parts, std::vector<int> ks, int max_iters, double tol,
                int min_iter, double rel_tol, int threads) {
    TORCH_CHECK(keys.scalar_type() == torch::kBFloat16 && keys.is_contiguous() && keys.dim() == 3);
    const int h = keys.size(0), n = keys.size(1), dim = keys.size(2);
    auto cfg = make_cfg(max_iters, tol, min_iter, rel_tol);
    std::unique_ptr<imi::KmeansResult> r;
    if (parts == 2) {
        r = imi::kmeans_execute(keys.data_ptr(), h, n, dim, ks[0], ks[1], torch::kBFloat16, threads, cfg);
    } else if (parts == 4) {
        r = imi::kmeans_execute_4(keys.data_ptr(), h, n, dim, ks[0], ks[1], ks[2], ks[3], torch::kBFloat16, threads, cfg);
    } else {
        r = imi::kmeans_execute_ivf(keys.data_ptr(), h, n, dim, ks[0], torch::kBFloat16, threads, cfg);
    }
    py::dict d;
    const int sub = parts == 0 ? dim : dim / parts;
    d["labels1"] = vec2d_i32(r->per_head_labels1, n);
    d["centroids1"] = vec2d_f32(r->per_head_centroids1, ks[0], sub);
    if (parts >= 2) {
        d["labels2"] = vec2d_i32(r->per_head_labels2, n);
        d["centroids2"] = vec2d_f32(r->per_head_centroids2, ks[1], sub);
    }
    if (parts == 4) {
        d["labels3"] = vec2d_i32(r->per_head_labels3, n);
        d["centroids3"] = vec2d_f32(r->per_head_centroids3, ks[2], sub);
        d["labels4"] = vec2d_i32(r->per_head_labels4, n);
        d["centroids4"] = vec2d_f32(r->per_head_centroids4, ks[3], sub);
    }
    std::vector<int32_t> ncl(r->per_head_n_clusters.begin(), r->per_head_n_clusters.end());
    d["n_clusters"] = torch::from_blob(ncl.data(), {h}, torch::kInt32).clone();
    return d;
}

// Full reference build: k-means + reorganize.  keys/values [h, n, dim] bf16.
py::dict build(torch::Tensor keys, torch::Tensor values, int parts, std::vector<int> ks, int max_iters,
               double tol, int min_iter, double rel_tol, int threads) {
    TORCH_CHECK(keys.scalar_type() == torch::kBFloat16 && keys.is_contiguous() && keys.dim() == 3);
    TORCH_CHECK(values.sizes() == keys.sizes() && values.is_contiguous());
    const int h = keys.size(0), n = keys.size(1), dim = keys.size(2);
    auto cfg = make_cfg(max_iters, tol, min_iter, rel_tol);
    std::unique_ptr<imi::KmeansResult> r;
    if (parts == 2) {
        r = imi::kmeans_execute(keys.data_ptr(), h, n, dim, ks[0], ks[1], torch::kBFloat16, threads, cfg);
    } else if (parts == 4) {
        r = imi::kmeans_execute_4(keys.data_ptr(), h, n, dim, ks[0], ks[1], ks[2], ks[3], torch::kBFloat16, threads, cfg);
    } else {
        r = imi::kmeans_execute_ivf(keys.data_ptr(), h, n, dim, ks[0], torch::kBFloat16, threads, cfg);
    }
    std::vector<imi::ReorganizeResult> out;
    std::vector<torch::Tensor> merged;
    if (parts == 2) {
        imi::reorganize_from_kmeans(keys, values, *r, n, dim / 2, out, merged, nullptr);
    } else if (parts == 4) {
        imi::reorganize_from_kmeans_4(keys, values, *r, n, dim / 4, out, merged, nullptr);
    } else {
        imi::reorganize_from_kmeans_ivf(keys, values, *r, n, out, merged, nullptr);
    }
    int64_t max_c = 0;
    for (auto& o : out) max_c = std::max<int64_t>(max_c, o.cluster_sizes.size());
    auto counts = torch::zeros({h}, torch::kInt32);
    auto sizes = torch::zeros({h, max_c}, torch::kInt32);
    auto offsets = torch::zeros({h, max_c + 1}, torch::kInt32);
    auto cents = torch::zeros({h, max_c, dim}, torch::kFloat32);
    auto rk = torch::empty({h, n, dim}, keys.options());
    auto rv = torch::empty({h, n, dim}, keys.options());
    for (int i = 0; i < h; ++i) {
        const int64_t c = out[i].cluster_sizes.size();
        counts[i] = static_cast<int32_t>(c);
        for (int64_t j = 0; j < c; ++j) sizes[i][j] = out[i].cluster_sizes[j];
        for (int64_t j = 0; j <= max_c; ++j)
            offsets[i][j] = out[i].cluster_offsets[std::min<int64_t>(j, c)];
        cents[i].narrow(0, 0, c).copy_(merged[i]);
        rk[i].copy_(out[i].reorganized_keys);
        rv[i].copy_(out[i].reorganized_values);
    }
    py::dict d;
    const int sub = parts == 0 ? dim : dim / parts;
    d["labels1"] = vec2d_i32(r->per_head_labels1, n);
    d["centroids1"] = vec2d_f32(r->per_head_centroids1, ks[0], sub);
    if (parts >= 2) {
        d["labels2"] = vec2d_i32(r->per_head_labels2, n);
        d["centroids2"] = vec2d_f32(r->per_head_centroids2, ks[1], sub);
    }
    if (parts == 4) {
        d["labels3"] = vec2d_i32(r->per_head_labels3, n);
        d["centroids3"] = vec2d_f32(r->per_head_centroids3, ks[2], sub);
        d["labels4"] = vec2d_i32(r->per_head_labels4, n);
        d["centroids4"] = vec2d_f32(r->per_head_centroids4, ks[3], sub);
    }
    d["cluster_counts"] = counts;
    d["cluster_sizes"] = sizes;
    d["cluster_offsets"] = offsets;
    d["centroids"] = cents;
    d["list_keys"] = rk;
    d["list_values"] = rv;
    return d;
}

}  // namespace

PYBIND11_MODULE(imi_ref, m) {
    m.def("kmeans", &kmeans, py::arg("keys"), py::arg("parts"), py::arg("ks"), py::arg("max_iters"),
          py::arg("tol"), py::arg("min_iter"), py::arg("rel_tol"), py::arg("threads") = 1);
    m.def("build", &build, py::arg("keys"), py::arg("values"), py::arg("parts"), py::arg("ks"),
          py::arg("max_iters"), py::arg("tol"), py::arg("min_iter"), py::arg("rel_tol"),
          py::arg("threads") = 1);
}
