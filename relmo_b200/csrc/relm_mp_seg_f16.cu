// Segment kernels instantiated for __half storage.
#include "relm_mp_seg_impl.cuh"

RELM_MP_INSTANTIATE(__half)
