// TVM-FFI export of the indexer: `launch_topk_c(q_index_fp8, k_index_cache_fp8,
// weights, seq_lens, block_table, topk_indices)`, destination-passing style,
// the signature of the reference entry point (solution/cuda/kernel.cu:818-824,
// bound through config.toml `entry_point = "kernel.cu::launch_topk_c"`). A
// tvm-ffi builder looks the symbol up by name; the stream comes from the
// TVM-FFI environment of the tensors' device. All work goes through the C ABI.
#include <dlpack/dlpack.h>
#include <tvm/ffi/container/tensor.h>
#include <tvm/ffi/error.h>
#include <tvm/ffi/extra/c_env_api.h>
#include <tvm/ffi/function.h>

#include <cstdint>

#include "dsa_topk_indexer.h"

namespace {

using tvm::ffi::TensorView;

bool compact(const TensorView& t) { return t.IsContiguous(); }

void require(bool ok, const char* what) {
  if (!ok) TVM_FFI_THROW(ValueError) << "launch_topk_c: " << what;
}

void LaunchTopkC(TensorView q, TensorView kc, TensorView w, TensorView sl, TensorView bt, TensorView out) {
  const DLDevice dev = q.device();
  require(dev.device_type == kDLCUDA, "tensors must be on a CUDA device");
  for (const TensorView* t : {&kc, &w, &sl, &bt, &out}) {
    require(t->device().device_type == dev.device_type && t->device().device_id == dev.device_id,
            "all tensors must be on the same device");
  }
  for (const TensorView* t : {&q, &kc, &w, &sl, &bt, &out}) require(compact(*t), "tensors must be contiguous");
  require(q.ndim() == 3 && q.size(1) == 64 && q.size(2) == 128 && q.dtype().bits == 8,
          "q_index_fp8 must be [B, 64, 128] fp8");
  const int64_t B = q.size(0);
  require(kc.ndim() >= 1 && kc.dtype().bits == 8 && kc.numel() == kc.size(0) * 8448,
          "k_index_cache_fp8 must be [num_pages, 64, 1, 132] bytes");
  require(w.ndim() == 2 && w.size(0) == B && w.size(1) == 64 && w.dtype().code == kDLFloat && w.dtype().bits == 32,
          "weights must be float32 [B, 64]");
  require(sl.ndim() == 1 && sl.size(0) == B && sl.dtype().code == kDLInt && sl.dtype().bits == 32,
          "seq_lens must be int32 [B]");
  require(bt.ndim() == 2 && bt.size(0) == B && bt.dtype().code == kDLInt && bt.dtype().bits == 32,
          "block_table must be int32 [B, max_num_pages]");
  require(out.ndim() == 2 && out.size(0) == B && out.size(1) == 2048 && out.dtype().code == kDLInt &&
              out.dtype().bits == 32,
          "topk_indices must be int32 [B, 2048]");
  int rc = dsa_topk_indexer_set_device(dev.device_id);
  if (rc == DSA_OK) {
    void* stream = TVMFFIEnvGetStream(dev.device_type, dev.device_id);
    rc = dsa_topk_indexer_launch(q.data_ptr(), kc.data_ptr(), static_cast<const float*>(w.data_ptr()),
                                 static_cast<const int32_t*>(sl.data_ptr()), static_cast<const int32_t*>(bt.data_ptr()),
                                 static_cast<int32_t*>(out.data_ptr()), B, bt.size(1), kc.size(0), stream);
  }
  if (rc != DSA_OK) TVM_FFI_THROW(RuntimeError) << "launch_topk_c: " << dsa_topk_indexer_error_string(rc);
}

}  // namespace

TVM_FFI_DLL_EXPORT_TYPED_FUNC(launch_topk_c, LaunchTopkC);
