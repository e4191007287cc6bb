// Segment kernels instantiated for float storage.
#include "relm_mp_seg_impl.cuh"

RELM_MP_INSTANTIATE(float)
