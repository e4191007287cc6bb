// Segment kernels instantiated for __nv_bfloat16 storage.
#include "relm_mp_seg_impl.cuh"

RELM_MP_INSTANTIATE(__nv_bfloat16)
