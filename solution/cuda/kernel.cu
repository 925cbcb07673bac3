// Entry translation unit of the harness solution slot
// `dsa_topk_indexer_fp8_h64_d128_topk2048_ps64` (config.toml:
// entry_point = "kernel.cu::launch_topk_c", destination-passing style), the
// slot the reference fills with solution/cuda/kernel.cu:818-891.
//
// The whole library is compiled into this one unit (dsa_indexer.cu and its
// headers sit beside this file in the packed solution, or on the include
// path when built from the repository). The binding depends on the builder:
//   - torch builder (torch.utils.cpp_extension defines TORCH_EXTENSION_NAME):
//     `launch_topk_c(torch::Tensor x6)` registered with PYBIND11_MODULE, on
//     the current torch stream, errors raised through TORCH_CHECK;
//   - tvm-ffi builder: the TVM_FFI_DLL_EXPORT_TYPED_FUNC export of
//     tvm_ffi_binding.cc.
// Both end in the C ABI dsa_topk_indexer_launch.
#if defined(TORCH_EXTENSION_NAME)
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#endif

#include "dsa_indexer.cu"

#if defined(TORCH_EXTENSION_NAME)

void launch_topk_c(torch::Tensor q_index_fp8, torch::Tensor k_index_cache_fp8, torch::Tensor weights,
                   torch::Tensor seq_lens, torch::Tensor block_table, torch::Tensor topk_indices) {
  const at::cuda::CUDAGuard guard(q_index_fp8.device());
  TORCH_CHECK(q_index_fp8.is_cuda() && q_index_fp8.dim() == 3 && q_index_fp8.size(1) == 64 &&
                  q_index_fp8.size(2) == 128 && q_index_fp8.element_size() == 1 && q_index_fp8.is_contiguous(),
              "q_index_fp8 must be a contiguous CUDA [B, 64, 128] fp8 tensor");
  const int64_t B = q_index_fp8.size(0);
  TORCH_CHECK(k_index_cache_fp8.element_size() == 1 && k_index_cache_fp8.is_contiguous() &&
                  k_index_cache_fp8.numel() == k_index_cache_fp8.size(0) * 8448,
              "k_index_cache_fp8 must be contiguous [num_pages, 64, 1, 132] bytes");
  TORCH_CHECK(weights.scalar_type() == torch::kFloat32 && weights.is_contiguous() && weights.size(0) == B &&
                  weights.size(1) == 64,
              "weights must be contiguous float32 [B, 64]");
  TORCH_CHECK(seq_lens.scalar_type() == torch::kInt32 && seq_lens.numel() == B && seq_lens.is_contiguous(),
              "seq_lens must be contiguous int32 [B]");
  TORCH_CHECK(block_table.scalar_type() == torch::kInt32 && block_table.dim() == 2 && block_table.size(0) == B &&
                  block_table.is_contiguous(),
              "block_table must be contiguous int32 [B, max_num_pages]");
  TORCH_CHECK(topk_indices.scalar_type() == torch::kInt32 && topk_indices.dim() == 2 && topk_indices.size(0) == B &&
                  topk_indices.size(1) == 2048 && topk_indices.is_contiguous(),
              "topk_indices must be contiguous int32 [B, 2048]");
  for (const torch::Tensor* t : {&k_index_cache_fp8, &weights, &seq_lens, &block_table, &topk_indices})
    TORCH_CHECK(t->device() == q_index_fp8.device(), "all tensors must be on the same device");
  const cudaStream_t stream = c10::cuda::getCurrentCUDAStream().stream();
  const int rc = dsa_topk_indexer_launch(q_index_fp8.data_ptr(), k_index_cache_fp8.data_ptr(),
                                         weights.data_ptr<float>(), seq_lens.data_ptr<int32_t>(),
                                         block_table.data_ptr<int32_t>(), topk_indices.data_ptr<int32_t>(), B,
                                         block_table.size(1), k_index_cache_fp8.size(0), stream);
  TORCH_CHECK(rc == DSA_OK, "launch_topk_c: ", dsa_topk_indexer_error_string(rc));
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("launch_topk_c", &launch_topk_c, "B200 DSA lightning-indexer top-2048 (destination-passing)");
}

#else
#include "tvm_ffi_binding.cc"
#endif
