// libkdb200.cu — the single translation unit of libkdb200.so.  Every kernel source is included here
// so that the device status word (kdb::g_status) is one symbol without relocatable device code.
#include "host_util.cu"
#include "proj.cu"
#include "moe_route.cu"
#include "moe_gemm.cu"
#include "moe_router_fast.cu"
#include "moe.cu"
#include "moe_ep.cu"
#include "moe_noalloc.cu"
#include "moe_w4a16.cu"
#include "selftest.cu"
#include "attention.cu"
#include "capi.cu"
