// Host-side schedule exports and the device range-bounds debug kernel.
#include <string.h>

#include <algorithm>

#include "common.cuh"

using namespace tc;

extern "C" int tc_version(void) { return 1; }

extern "C" int64_t tc_launch_count(void) { return launch_counter().load(); }

static int fill_schedule(const int32_t* act, int nl, int32_t cache, int32_t n, tc_schedule* out) {
  if (nl < 1 || nl > TC_MAX_LEVELS || cache <= 0 || n <= 0 || act[0] != 0) return TC_ERR_ARG;
  memset(out, 0, sizeof(*out));
  out->num_levels = nl;
  out->cache_size = cache;
  out->seq_len = n;
  int64_t off = 0;
  for (int l = 0; l < nl; ++l) {
    out->act[l] = act[l];
    out->level_len[l] = n >> l;
    out->offsets[l] = off;
    off += n >> l;
  }
  out->offsets[nl] = off;
  // Coarsest lifetime span (range_spec.py:287-317): sweep q, evicting the
  // coarsest nodes older than the raw oldest node; the longest lifetime of a
  // node born before N is the constant bwd hulls add; N if nothing is evicted.
  const int top = nl - 1;
  const int n_nodes = n >> top;
  int lo[TC_MAX_LEVELS], hi[TC_MAX_LEVELS];
  int64_t span = 0;
  int evicted = 0;
  for (int q = 0; q < n; ++q) {
    row_bounds_raw(q, act, nl, cache, lo, hi);
    while (evicted < lo[top] && evicted < n_nodes) {
      const int64_t born = (int64_t)act[top] + ((int64_t)evicted << top);
      if (born < n) span = std::max<int64_t>(span, q - born);
      ++evicted;
    }
  }
  out->coarsest_span = span ? (int32_t)span : n;
  return TC_OK;
}

extern "C" int tc_schedule_from_times(const int32_t* act, int32_t num_levels, int32_t cache_size,
                                      int32_t seq_len, tc_schedule* out) {
  if (!act || !out) return TC_ERR_ARG;
  return fill_schedule(act, num_levels, cache_size, seq_len, out);
}

extern "C" int tc_schedule_init(const int32_t* fmap_vals, int32_t L, int32_t cache_size,
                                int32_t seq_len, tc_schedule* out) {
  if (!out || L < 0 || L + 1 > TC_MAX_LEVELS || (L > 0 && !fmap_vals)) return TC_ERR_ARG;
  int32_t act[TC_MAX_LEVELS] = {0};
  // activation_times_from_fmap (range_spec.py:26-54)
  if (L >= 1) act[1] = fmap_vals[0] + 1;
  for (int l = 2; l <= L; ++l)
    act[l] = act[l - 1] + (1 << (l - 1)) * (fmap_vals[l - 1] - fmap_vals[l - 2]) + (1 << (l - 2));
  for (int l = 1; l <= L; ++l) {
    const int ph = ((act[l] % (1 << l)) + (1 << l)) % (1 << l);
    if (ph != (1 << (l - 1))) return TC_ERR_SCHEDULE;
  }
  return fill_schedule(act, L + 1, cache_size, seq_len, out);
}

extern "C" int tc_schedule_stats(const tc_schedule* s, int64_t* out3) {
  if (!s || !out3) return TC_ERR_ARG;
  const Sched d = make_sched(*s);
  int lo[TC_MAX_LEVELS], hi[TC_MAX_LEVELS];
  int64_t mn = INT64_MAX, mx = 0, tot = 0;
  for (int q = 0; q < d.n; ++q) {
    const int m = row_bounds(q, d, lo, hi);
    mn = std::min<int64_t>(mn, m);
    mx = std::max<int64_t>(mx, m);
    tot += m;
  }
  out3[0] = mn;
  out3[1] = mx;
  out3[2] = tot;
  return TC_OK;
}

extern "C" int tc_decode_caps(const int32_t* act, int32_t nl, int32_t cache, int32_t* caps) {
  // Peak live count per level over two schedule periods past the last
  // activation (reference.py:1739-1772).
  if (!act || !caps || nl < 1 || nl > TC_MAX_LEVELS || cache <= 0 || act[0] != 0) return TC_ERR_ARG;
  const int top = nl - 1;
  const int64_t horizon = 2 * ((int64_t)act[top] + (1LL << (top + 1))) + 1;
  tc_schedule s;
  int rc = fill_schedule(act, nl, cache, (int32_t)std::min<int64_t>(horizon, INT32_MAX), &s);
  if (rc) return rc;
  const Sched d = make_sched(s);
  for (int l = 0; l < nl; ++l) caps[l] = 0;
  int lo[TC_MAX_LEVELS], hi[TC_MAX_LEVELS];
  for (int64_t q = 0; q < horizon; ++q) {
    row_bounds((int)q, d, lo, hi);
    int used = 0;
    for (int l = 0; l < top; ++l) {
      caps[l] = std::max(caps[l], hi[l] - lo[l]);
      used += hi[l] - lo[l];
    }
    if (used > cache) return TC_ERR_ARG;
    caps[top] = std::max(caps[top], cache - used);
  }
  return TC_OK;
}

extern "C" int tc_range_bounds_host(const tc_schedule* s, const int32_t* qs, int32_t n, int32_t* out) {
  if (!s || (n > 0 && (!qs || !out))) return TC_ERR_ARG;
  const Sched d = make_sched(*s);
  int lo[TC_MAX_LEVELS], hi[TC_MAX_LEVELS];
  for (int i = 0; i < n; ++i) {
    if (qs[i] < 0 || qs[i] >= d.n) return TC_ERR_ARG;
    row_bounds(qs[i], d, lo, hi);
    for (int l = 0; l < d.nl; ++l) {
      out[(i * d.nl + l) * 2] = lo[l];
      out[(i * d.nl + l) * 2 + 1] = hi[l];
    }
  }
  return TC_OK;
}

extern "C" int tc_hulls_host(const tc_schedule* s, int32_t kind, int32_t level, const int32_t* lo,
                             const int32_t* hi, int32_t n, int32_t* out) {
  if (!s || level < 0 || level >= s->num_levels || (n > 0 && (!lo || !hi || !out))) return TC_ERR_ARG;
  const Sched d = make_sched(*s);
  for (int i = 0; i < n; ++i) {
    int a = 0, b = 0;
    if (kind == 0) {
      if (lo[i] < 0 || lo[i] > hi[i] || hi[i] > d.n) return TC_ERR_ARG;
      fwd_hull(lo[i], hi[i], level, d, &a, &b);
    } else {
      if (lo[i] < 0 || lo[i] > hi[i] || hi[i] > d.len[level]) return TC_ERR_ARG;
      bwd_hull(lo[i], hi[i], level, d, &a, &b);
    }
    out[2 * i] = a;
    out[2 * i + 1] = b;
  }
  return TC_OK;
}

__global__ void range_bounds_kernel(Sched d, const int32_t* qs, int32_t n, int32_t* out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  int lo[TC_MAX_LEVELS], hi[TC_MAX_LEVELS];
  const int q = qs[i];
  if (q < 0 || q >= d.n) {
    for (int l = 0; l < d.nl; ++l) out[(i * d.nl + l) * 2] = out[(i * d.nl + l) * 2 + 1] = -1;
    return;
  }
  row_bounds(q, d, lo, hi);
  for (int l = 0; l < d.nl; ++l) {
    out[(i * d.nl + l) * 2] = lo[l];
    out[(i * d.nl + l) * 2 + 1] = hi[l];
  }
}

extern "C" int tc_range_bounds_device(const tc_schedule* s, const int32_t* qs, int32_t n, int32_t* out,
                                      void* stream) {
  if (!s || n < 0 || (n > 0 && (!qs || !out))) return TC_ERR_ARG;
  if (n == 0) return TC_OK;
  range_bounds_kernel<<<(n + 127) / 128, 128, 0, (cudaStream_t)stream>>>(make_sched(*s), qs, n, out);
  return launch_status();
}
