// Segment kernels instantiated for double storage.
#include "relm_mp_seg_impl.cuh"

RELM_MP_INSTANTIATE(double)
