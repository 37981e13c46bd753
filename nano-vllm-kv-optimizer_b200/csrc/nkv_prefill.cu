// Kernel (4): segmented prefill attention (tcgen05/TMEM).  Placeholder entry
// points until the tensor-core kernel lands: they reject every call.
#include "nkv_common.cuh"
#include "nkv_host.h"

extern "C" size_t nkv_prefill_workspace_bytes(int hkv, int hq, int nq, int max_tokens) {
  (void)hkv; (void)hq; (void)nq; (void)max_tokens;
  return 256;
}

extern "C" int nkv_prefill(nkv_stream_t stream, const nkv_attend_args* a) {
  (void)stream; (void)a;
  nkv::set_error("prefill: tensor-core kernel not built in this version");
  return NKV_ERR_UNSUPPORTED;
}
