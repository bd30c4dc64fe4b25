// Single translation unit for libfa_b200.so: the kernels share the
// device-side error word, which (without relocatable device code) must be
// defined in the same unit that uses it.
#include "capi.cu"
#include "decode_sm100.cu"
#include "decode_d128_sm100.cu"
#include "decode_gqa_sm100.cu"
#include "prefill_sm100.cu"
#include "prefill_d128_sm100.cu"
#include "legacy_sm100.cu"
#include "noalloc.cu"
#include "host_stage.cu"
