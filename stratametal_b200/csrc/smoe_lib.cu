// smoe_lib.cu - the library's single translation unit: every kernel file and the C ABI are compiled here
// together, so the per-device status word (common.cuh) is one symbol without relocatable device code.
#include "router.cu"
#include "dispatch.cu"
#include "expert.cu"
#include "combine.cu"
#include "tc.cu"
#include "tq.cu"
#include "iqx.cu"
#include "elementwise.cu"
#include "decode.cu"
#include "ep.cu"
#include "api.cu"
#include "noalloc.cu"
