// Helpers shared by the binding translation units (torch side only).
#pragma once
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

namespace afb_bind {
uint32_t* status_ptr(int dev);  // defined in bindings.cpp
inline cudaStream_t stream() { return at::cuda::getCurrentCUDAStream().stream(); }
inline void check_rc(int rc, const char* what) { TORCH_CHECK(rc == 0, what, " failed with code ", rc); }
int num_sms();
template <class T>
inline T* ptr(const at::Tensor& t) {
  return reinterpret_cast<T*>(t.data_ptr());
}
template <class T>
inline T* optr(const c10::optional<at::Tensor>& t) {
  return t.has_value() && t->defined() ? reinterpret_cast<T*>(t->data_ptr()) : nullptr;
}
}  // namespace afb_bind

#define AFB_CHECK_CUDA(x) TORCH_CHECK((x).is_cuda(), #x " must be a CUDA tensor")
#define AFB_CHECK_DT(x, dt) \
  TORCH_CHECK((x).scalar_type() == (dt), #x " has dtype ", (x).scalar_type(), ", expected ", dt)
#define AFB_CHECK_CONTIG(x) TORCH_CHECK((x).is_contiguous(), #x " must be contiguous")
