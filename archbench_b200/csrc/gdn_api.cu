// C-ABI entry points (include/gdn_b200.h): argument validation and kernel selection.
// Nothing here allocates device memory or synchronises the stream.
#include <string.h>

#include "gdn_common.cuh"

namespace {

int dtype_size(int dt) {
  switch (dt) {
    case GDN_DTYPE_F32: return 4;
    case GDN_DTYPE_BF16: return 2;
    default: return 0;
  }
}

// The current device must be an sm_100 part: the library carries sm_100a code only.
int check_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return GDN_ERR_DEVICE;
  static std::atomic<int> cached[64] = {};  // 0 unknown, 1 ok, -1 bad (any host thread may call)
  if (dev >= 0 && dev < 64) {
    const int c = cached[dev].load(std::memory_order_relaxed);
    if (c != 0) return c > 0 ? GDN_OK : GDN_ERR_DEVICE;
  }
  int major = 0, minor = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess)
    return GDN_ERR_DEVICE;
  const bool ok = (major == 10 && minor == 0);
  if (dev >= 0 && dev < 64) cached[dev].store(ok ? 1 : -1, std::memory_order_relaxed);
  return ok ? GDN_OK : GDN_ERR_DEVICE;
}

bool aligned(const void* p, int bytes) { return ((uintptr_t)p % (uintptr_t)bytes) == 0; }

bool strides_ok(const gdn_strides& s, int64_t elem, int vec_bytes) {
  auto ok = [&](int64_t x) { return x >= 0 && (x * elem) % vec_bytes == 0; };
  return ok(s.b) && ok(s.t) && ok(s.h);
}

// Validation shared by prefill and decode.  `T` may be 0.
int validate(const gdn_prefill_args* a) {
  if (!a) return GDN_ERR_NULL;
  if (a->B <= 0 || a->H <= 0 || a->T < 0) return GDN_ERR_SHAPE;
  // With T == 0 no token tensor is read or written (empty tensors may have NULL data).
  if (a->T > 0) {
    if (!a->q || !a->k || !a->v || !a->la || !a->y) return GDN_ERR_NULL;
    if (!a->u && !a->beta) return GDN_ERR_NULL;
  }
  if (!(a->DK == 32 || a->DK == 64 || a->DK == 128 || a->DK == 256)) return GDN_ERR_UNSUPPORTED;
  if (a->DV < 1 || a->DV > 1024) return GDN_ERR_UNSUPPORTED;
  if (a->B > (1 << 20) || a->H > (1 << 16) || a->T > (1LL << 31) - 1) return GDN_ERR_SHAPE;
  if (a->B * a->H * a->DV > (1LL << 31)) return GDN_ERR_SHAPE;
  const int es = dtype_size(a->in_dtype);
  if (!es || !dtype_size(a->out_dtype)) return GDN_ERR_DTYPE;
  if (a->impl < GDN_IMPL_AUTO || a->impl > GDN_IMPL_CHUNK_SPLIT) return GDN_ERR_UNSUPPORTED;
  // The recurrent kernel reads DK/32 consecutive elements per lane as one vector.
  const int vec = (int)(a->DK / 32) * es;
  const int vb = vec >= 16 ? 16 : vec;
  if (!aligned(a->q, vb) || !aligned(a->k, vb) || (a->u && !aligned(a->u, vb))) return GDN_ERR_ALIGN;
  if (!strides_ok(a->sq, es, vb) || !strides_ok(a->sk, es, vb) || (a->u && !strides_ok(a->su, es, vb)))
    return GDN_ERR_ALIGN;
  if (!aligned(a->v, es) || !aligned(a->y, dtype_size(a->out_dtype))) return GDN_ERR_ALIGN;
  if (!strides_ok(a->sv, es, es) || !strides_ok(a->sy, dtype_size(a->out_dtype), dtype_size(a->out_dtype)))
    return GDN_ERR_ALIGN;
  const int svec = (int)(a->DK / 32) * 4 >= 16 ? 16 : (int)(a->DK / 32) * 4;
  if ((a->s0 && !aligned(a->s0, svec)) || (a->s_out && !aligned(a->s_out, svec))) return GDN_ERR_ALIGN;
  return GDN_OK;
}

// SM count used for planning: the current device's when a CUDA device is present, else the
// B200's 148 (host-only queries on machines without a GPU).
int plan_sms() {
  const int n = gdn_segmented_sms();
  return n > 0 ? n : 148;
}

// The chunk variant for these arguments: the two-CTA cluster kernel where it applies (DV = 128,
// u = beta k), else the single-CTA kernel.
int chunk_variant(const gdn_prefill_args* a) {
  return (a->u == nullptr && gdn_chunk_pair_supported(a)) ? (int)GDN_IMPL_CHUNK_CLUSTER : (int)GDN_IMPL_CHUNK_SINGLE;
}

// The segmented path pays for a state pass over all but the last segment; it beats the cluster
// kernel only when the sequences are so few that the cluster kernel leaves most SMs idle (fewer
// than one (b, h) unit per 8 SMs).  Where the cluster kernel does not apply, the plan decides.
bool segmented_preferred(const gdn_prefill_args* a, int sms) {
  if (chunk_variant(a) != GDN_IMPL_CHUNK_CLUSTER) return true;
  return a->B * a->H * 8 <= (int64_t)sms;
}

// Waves of CTAs a launch of `ctas` CTAs takes at `per_wave` resident at once.
int64_t waves(int64_t ctas, int64_t per_wave) { return per_wave > 0 ? (ctas + per_wave - 1) / per_wave : ctas; }

// The split path (prep pass over every chunk, then the state-only chunk kernel: one CTA per sequence
// and 128-row state slice) where the cluster kernel does not apply -- state rows beyond 128 or
// explicit write vectors -- or where the cluster kernel, two SMs per sequence, would need more waves
// than the state-only kernel (more sequences than clusters fit on the GPU).  Its workspace holds
// every chunk's products.
bool split_preferred(const gdn_prefill_args* a) {
  if (!gdn_chunk_supported(a) || !gdn_chunk_split_supported(a)) return false;
  if (chunk_variant(a) != GDN_IMPL_CHUNK_CLUSTER) return true;
  const int clusters = gdn_chunk_pair_max_clusters();
  const int64_t seqs = a->B * a->H;
  return clusters > 0 && waves(seqs, clusters) > waves(seqs, plan_sms());
}

int select_impl(const gdn_prefill_args* a) {
  const bool chunk_ok = gdn_chunk_supported(a);
  int P = 0, L = 0;
  size_t need = 0;
  const bool seg_ok = chunk_ok && gdn_segmented_plan(a, plan_sms(), &P, &L, &need);
  const bool seg_auto = seg_ok && segmented_preferred(a, plan_sms());
  const bool ws_ok = seg_ok && a->workspace != nullptr && a->workspace_bytes >= need;
  const bool split_ok = chunk_ok && gdn_chunk_split_supported(a);
  const bool split_ws = split_ok && a->workspace != nullptr && a->workspace_bytes >= gdn_chunk_prep_bytes(a);
  switch (a->impl) {
    case GDN_IMPL_CHUNK: return chunk_ok ? chunk_variant(a) : (int)GDN_ERR_UNSUPPORTED;
    case GDN_IMPL_CHUNK_CLUSTER:
      return chunk_ok && chunk_variant(a) == GDN_IMPL_CHUNK_CLUSTER ? (int)GDN_IMPL_CHUNK_CLUSTER
                                                                     : (int)GDN_ERR_UNSUPPORTED;
    case GDN_IMPL_CHUNK_SINGLE: return chunk_ok ? (int)GDN_IMPL_CHUNK_SINGLE : (int)GDN_ERR_UNSUPPORTED;
    case GDN_IMPL_RECURRENT: return (int)GDN_IMPL_RECURRENT;
    case GDN_IMPL_SEGMENTED:
      if (!seg_ok) return (int)GDN_ERR_UNSUPPORTED;
      return ws_ok ? (int)GDN_IMPL_SEGMENTED : (int)GDN_ERR_SHAPE;
    case GDN_IMPL_CHUNK_SPLIT:
      if (!split_ok) return (int)GDN_ERR_UNSUPPORTED;
      return split_ws ? (int)GDN_IMPL_CHUNK_SPLIT : (int)GDN_ERR_SHAPE;
    default:
      if (ws_ok && seg_auto) return (int)GDN_IMPL_SEGMENTED;
      if (split_ws && split_preferred(a)) return (int)GDN_IMPL_CHUNK_SPLIT;
      return chunk_ok ? chunk_variant(a) : (int)GDN_IMPL_RECURRENT;
  }
}

}  // namespace

extern "C" {

int gdn_abi_version(void) { return GDN_B200_ABI_VERSION; }

const char* gdn_status_string(int s) {
  switch (s) {
    case GDN_OK: return "ok";
    case GDN_ERR_NULL: return "a required pointer is NULL";
    case GDN_ERR_SHAPE: return "a size is out of range or inconsistent";
    case GDN_ERR_DTYPE: return "unsupported dtype";
    case GDN_ERR_ALIGN: return "pointer or stride misaligned for the kernel's vector accesses";
    case GDN_ERR_UNSUPPORTED: return "no kernel of this build implements this request";
    case GDN_ERR_DEVICE: return "the current device is not an sm_100 (B200) GPU";
    case GDN_ERR_LAUNCH: return "CUDA kernel launch failed";
    case GDN_ERR_TIMEOUT: return "a bounded device-side wait gave up";
    case GDN_ERR_WORKSPACE: return "the problem needs more segment scratch than GDN_STATIC_WORKSPACE_BYTES";
    default: return "unknown gdn_status";
  }
}

int gdn_device_status(int* status, int reset) {
  if (!status) return GDN_ERR_NULL;
  int st = check_device();
  if (st != GDN_OK) return st;
  int single = 0, pair = 0, prep = 0;
  st = gdn_chunk_read_status(&single, reset);
  if (st != GDN_OK) return st;
  st = gdn_chunk_pair_read_status(&pair, reset);
  if (st != GDN_OK) return st;
  st = gdn_chunk_prep_read_status(&prep, reset);
  if (st != GDN_OK) return st;
  *status = single != 0 ? single : (pair != 0 ? pair : prep);
  return GDN_OK;
}

int gdn_selftest_bounded_wait(long long max_cycles, void* stream) {
  int st = check_device();
  if (st != GDN_OK) return st;
  return gdn_launch_selftest_wait(max_cycles, static_cast<cudaStream_t>(stream));
}

int gdn_prefill_workspace_bytes(const gdn_prefill_args* a, size_t* bytes) {
  if (!bytes) return GDN_ERR_NULL;
  int st = validate(a);
  if (st != GDN_OK) return st;
  *bytes = 0;
  int P = 0, L = 0;
  size_t need = 0;
  if ((a->impl == GDN_IMPL_SEGMENTED || (a->impl == GDN_IMPL_AUTO && gdn_chunk_supported(a) &&
                                           segmented_preferred(a, plan_sms()))) &&
      a->T > 0 && gdn_segmented_plan(a, plan_sms(), &P, &L, &need))
    *bytes = need;
  else if (a->T > 0 && ((a->impl == GDN_IMPL_CHUNK_SPLIT && gdn_chunk_supported(a) && gdn_chunk_split_supported(a)) ||
                        (a->impl == GDN_IMPL_AUTO && split_preferred(a))))
    *bytes = gdn_chunk_prep_bytes(a);
  return GDN_OK;
}

int gdn_prefill_select_impl(const gdn_prefill_args* a) {
  int st = validate(a);
  if (st != GDN_OK) return st;
  return select_impl(a);
}

int gdn_prefill_fwd(const gdn_prefill_args* a, void* stream) {
  int st = validate(a);
  if (st != GDN_OK) return st;
  st = check_device();
  if (st != GDN_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (a->T == 0) {  // nothing to scan: S_T = S_0
    if (a->s_out && a->s_out != a->s0) {
      const size_t n = (size_t)(a->B * a->H * a->DV * a->DK) * sizeof(float);
      cudaError_t e = a->s0 ? cudaMemcpyAsync(a->s_out, a->s0, n, cudaMemcpyDeviceToDevice, s)
                            : cudaMemsetAsync(a->s_out, 0, n, s);
      if (e != cudaSuccess) return GDN_ERR_LAUNCH;
    }
    return GDN_OK;
  }
  const int impl = select_impl(a);
  if (impl < 0) return impl;
  if (impl == GDN_IMPL_SEGMENTED)
    return gdn_launch_segmented(a, static_cast<float*>(a->workspace), (size_t)a->workspace_bytes, plan_sms(), s);
  if (impl == GDN_IMPL_CHUNK_CLUSTER) return gdn_launch_chunk_pair(a, 1, 0, nullptr, 0, s);
  if (impl == GDN_IMPL_CHUNK_SPLIT) {
    st = gdn_launch_chunk_prep(a, a->workspace, s);
    if (st != GDN_OK) return st;
    return gdn_launch_chunk_split(a, a->workspace, 0, 1, 0, nullptr, 0, s);
  }
  if (impl == GDN_IMPL_CHUNK_SINGLE) return gdn_launch_chunk_sm100(a, s);
  return gdn_launch_recurrent(a, a->s0, a->s_out, s);
}

int gdn_prefill_fwd_static_workspace(const gdn_prefill_args* a, void* stream) {
  if (!a) return GDN_ERR_NULL;
  gdn_prefill_args checked = *a;  // impl is ignored by this entry point, so it is not validated
  checked.impl = GDN_IMPL_AUTO;
  int st = validate(&checked);
  if (st != GDN_OK) return st;
  st = check_device();
  if (st != GDN_OK) return st;
  if (a->T == 0) return GDN_ERR_UNSUPPORTED;
  return gdn_launch_segmented_static(&checked, plan_sms(), static_cast<cudaStream_t>(stream));
}

int gdn_decode_step(const gdn_decode_args* d, void* stream) {
  if (!d) return GDN_ERR_NULL;
  if (!d->state) return GDN_ERR_NULL;
  gdn_prefill_args a;
  memset(&a, 0, sizeof(a));
  a.q = d->q; a.k = d->k; a.u = d->u; a.v = d->v;
  a.beta = d->beta; a.la = d->la; a.s0 = d->state; a.s_out = d->state; a.y = d->y;
  a.sq = d->sq; a.sk = d->sk; a.su = d->su; a.sv = d->sv; a.sy = d->sy;
  a.sq.t = a.sk.t = a.su.t = a.sv.t = a.sy.t = 0;  // one token: the t stride is never used
  a.B = d->B; a.T = 1; a.H = d->H; a.DK = d->DK; a.DV = d->DV;
  a.in_dtype = d->in_dtype; a.out_dtype = d->out_dtype; a.impl = GDN_IMPL_RECURRENT;
  int st = validate(&a);
  if (st != GDN_OK) return st;
  st = check_device();
  if (st != GDN_OK) return st;
  return gdn_launch_recurrent(&a, d->state, d->state, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
