// Chunkwise-parallel gated delta rule on tcgen05 / TMEM (sm_100a).  (placeholder)
#include "gdn_common.cuh"

bool gdn_chunk_supported(const gdn_prefill_args* a) { (void)a; return false; }
int gdn_launch_chunk_sm100(const gdn_prefill_args* a, cudaStream_t stream) {
  (void)a; (void)stream;
  return GDN_ERR_UNSUPPORTED;
}
