// Argument checks shared by the CUDA and CPU registrations of torch.ops.relm_mp
// (relm_mp_torch.cpp, relm_mp_cpu.cpp). Their messages are the reference's
// error contract (mp_ops.cpp:38-71), which callers and tests match on.
#pragma once

#include <ATen/ATen.h>

namespace relm_b200 {

void check_rank(const at::Tensor& t, int64_t expected, const char* name);
void check_int64_index(const at::Tensor& t, const char* name);
void check_int32_or_int64_index(const at::Tensor& t, const char* name);
at::Tensor contig(const at::Tensor& t);

}  // namespace relm_b200
