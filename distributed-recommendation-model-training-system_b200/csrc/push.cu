// push.cu -- gradient push: coalesced segment-sum fused with the row-wise sparse
// LazyAdam update, with the reference's all-or-nothing rejection.
//
// Reference semantics followed:
//   * src/access/batch_access.cpp:89-123 (ReduceGradients): every gradient value
//     must be finite; per table, each unique row receives
//     g += src_row * scale over its occurrences in (feature, bag, position) order,
//     scale = 1.0f/valid_length for mean; a non-finite reduced value rejects.
//   * src/update/lazy_adam.cpp:7-42 (ValidateLazyAdam / ApplyLazyAdam):
//     lr_t = lr*sqrt(1-b2p)/(1-b1p) in float; m = b1*m + (1-b1)*g;
//     v = b2*v + (1-b2)*g*g; w -= lr_t*m/(sqrt(v)+eps); clamp; ++updates; then
//     ++optimizer_sequence, b1p *= b1, b2p *= b2 per table.
//   * src/server/service.cpp:252-325: all tables are validated before any is
//     written; a rejected Push leaves every byte of state unchanged.
//
// Launch sequence (all decisions are made on the device; no host sync):
//   1. prescan   -- finiteness + max|g| of every gradient value; its last block
//                   computes lr_t per table and picks the mode:
//                   SAFE    when |g_reduced| <= 3*N*max|g| <= 1e17, the recorded
//                           state bound <= 1e17 and lr_t/eps <= 1e20: then no
//                           m, v or w can overflow (|lr_t*m/(sqrt(v)+eps)| <=
//                           1e37) and the update is applied in ONE fused pass;
//                   CHECKED otherwise: pass 0 validates exactly as the reference,
//                           pass 1 applies only if nothing was rejected.
//   2. segments pass 0, 3. long pass 0, 4. segments pass 1, 5. long pass 1,
//   6. finalize  -- advances beta powers and the sequence iff accepted.
//
// Coalescing layout: the occurrences are sorted stably by composite key
// (table rank, slot).  A group of G lanes (G = D/4: one 128-bit access per lane
// covers a row) owns the tile [32t, 32t+32) of sorted occurrences and fully
// processes every segment that STARTS in its tile and has at most 64
// occurrences: the row's state load is issued first, the gradient sum runs
// serially in occurrence order (bit-exact with the reference) with up to 8
// gradient rows in flight, and the Adam update of that row follows in the same
// pass.  Longer (Zipf-head) segments are reduced per tile into part0/part1 and
// combined in tile order by all groups of one CTA in the long-segment kernel
// (deterministic; within 1e-6 * sum|terms| of the reference's serial sum).
#include <cooperative_groups.h>
#include <cooperative_groups/reduce.h>

#include "kernels.cuh"

namespace cg = cooperative_groups;

namespace eps_b200 {
namespace {

template <typename KeyT>
__device__ __forceinline__ KeyT key_at(const void* keys, unsigned long long i) {
  return __ldg(static_cast<const KeyT*>(keys) + i);
}

struct Role { bool run, apply, validate, partials; };

__device__ __forceinline__ Role role(const PushControl* c, int pass) {
  Role r{false, false, false, false};
  const unsigned mode = *(volatile const unsigned*)&c->mode;
  if (mode == kModeRejected) return r;
  if (pass == 0) {
    r.run = true; r.partials = true;
    r.apply = mode == kModeSafe;
    r.validate = mode == kModeChecked;
  } else {
    const unsigned bits = *(volatile const unsigned*)&c->reject_bits;
    if (mode != kModeChecked || bits) return r;
    r.run = true; r.apply = true;
  }
  return r;
}

// ------------------------------------------------------------------ prescan
__global__ void __launch_bounds__(256) push_prescan(PushLaunch p, PushTable* tables_rw) {
  __shared__ unsigned long long s_prefix[kMaxFeatures + 1];
  __shared__ unsigned s_bad, s_max, s_last;
  const unsigned fc = p.feature_count;
  for (unsigned i = threadIdx.x; i <= fc; i += blockDim.x) s_prefix[i] = p.grad_prefix[i];
  if (threadIdx.x == 0) { s_bad = 0; s_max = 0; }
  __syncthreads();
  const unsigned long long total = p.grad_values;
  const unsigned long long per_block = (total + gridDim.x - 1) / gridDim.x;
  const unsigned long long begin = min(total, per_block * blockIdx.x);
  const unsigned long long end = min(total, begin + per_block);
  unsigned bad = 0;
  float mx = 0.0f;
  unsigned f = 0;
  {  // feature containing `begin`
    unsigned lo = 0, hi = fc;
    while (hi - lo > 1) { const unsigned mid = (lo + hi) >> 1; if (s_prefix[mid] <= begin) lo = mid; else hi = mid; }
    f = lo;
  }
  for (unsigned long long i = begin + threadIdx.x; i < end; i += blockDim.x) {
    while (f + 1 < fc && s_prefix[f + 1] <= i) ++f;
    const float x = __ldg(p.features[f].grad + (i - s_prefix[f]));
    bad |= !isfinite(x);
    mx = fmaxf(mx, fabsf(x));
  }
  bad = __reduce_or_sync(0xffffffffu, bad);
  unsigned mb = __reduce_max_sync(0xffffffffu, __float_as_uint(mx));
  if ((threadIdx.x & 31) == 0) {
    if (bad) atomicOr(&s_bad, 1u);
    atomicMax(&s_max, mb);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    if (s_bad) atomicOr(&p.control->nonfinite, 1u);
    atomicMax(&p.control->maxabs_bits, s_max);
    __threadfence();
    s_last = atomicAdd(&p.control->blocks_done, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!s_last || threadIdx.x != 0) return;
  __threadfence();
  // ---- decision (single thread of the last block)
  PushControl* c = p.control;
  unsigned bits = 0;
  const unsigned lookup_err = *(volatile const unsigned*)p.lookup_error;
  if (lookup_err) { c->reject_bits = 16u; c->mode = kModeRejected; return; }
  if (*(volatile unsigned*)&c->nonfinite) { c->reject_bits = kRejectNonFiniteInput; c->mode = kModeRejected; return; }
  const float maxabs = __uint_as_float(*(volatile unsigned*)&c->maxabs_bits);
  bool safe = true;
  for (unsigned t = 0; t < p.table_count; ++t) {
    PushTable& T = tables_rw[t];
    const float b1p = T.dtable->beta1_power, b2p = T.dtable->beta2_power;
    // src/update/lazy_adam.cpp:27 -- (lr * sqrt(1 - b2p)) / (1 - b1p)
    const float lr_t = __fdiv_rn(__fmul_rn(T.learning_rate, __fsqrt_rn(__fsub_rn(1.0f, b2p))),
                                 __fsub_rn(1.0f, b1p));
    T.lr_t = lr_t;
    if (!isfinite(lr_t)) bits |= kRejectLearningRate;
    const double G = 3.0 * (double)T.occurrences * (double)maxabs;
    const double A = (double)__uint_as_float(T.dtable->state_absmax_bits);
    if (!(G <= 1e17 && A <= 1e17 && (double)lr_t <= 1e20 * (double)T.epsilon)) safe = false;
  }
  c->reject_bits = bits;
  c->mode = (safe && !bits) ? kModeSafe : kModeChecked;
  __threadfence();
}

// ------------------------------------------------------ reduction helpers
template <int G>
__device__ __forceinline__ unsigned full_mask() { return G == 32 ? 0xffffffffu : ((1u << G) - 1u); }

// Sum of gradient references [s0, s1) (all with the same key), serially in order,
// by the G lanes of `grp` (each lane owns VEC*ITERS columns).
template <int G, int VEC, int ITERS, typename Grp>
__device__ __forceinline__ void accumulate_global(const Grp& grp, const PushLaunch& p,
                                                  unsigned long long s0, unsigned long long s1,
                                                  unsigned D, float (&acc)[VEC * ITERS]) {
  constexpr int C = VEC * ITERS;
  constexpr int DEPTH = C <= 4 ? 4 : 2;
  const unsigned gl = grp.thread_rank();
  for (unsigned long long c0 = s0; c0 < s1; c0 += G) {
    const unsigned long long i = c0 + gl;
    unsigned long long gp = 0;
    float sc = 0.0f;
    if (i < s1) {
      const unsigned src = __ldg(p.srcs + i);
      const unsigned f = src >> kRowBits;
      const unsigned r = src & ((1u << kRowBits) - 1u);
      const PushFeature* F = p.features + f;
      const float* g = reinterpret_cast<const float*>(__ldg(reinterpret_cast<const unsigned long long*>(&F->grad)));
      gp = reinterpret_cast<unsigned long long>(g + (unsigned long long)r * D);
      sc = __ldg(p.row_scale + __ldg(&F->scale_base) + r);
    }
    const int cnt = (int)min((unsigned long long)G, s1 - c0);
    for (int j0 = 0; j0 < cnt; j0 += DEPTH) {
      float x[DEPTH][C];
      float s[DEPTH];
#pragma unroll
      for (int u = 0; u < DEPTH; ++u) {
        const unsigned long long q = grp.shfl(gp, (j0 + u) & (G - 1));
        s[u] = grp.shfl(sc, (j0 + u) & (G - 1));
        const bool use = j0 + u < cnt;
#pragma unroll
        for (int it = 0; it < ITERS; ++it) {
          const unsigned col = (it * G + gl) * VEC;
          float t[VEC];
          if (use && col < D) load_vec<VEC>(reinterpret_cast<const float*>(q) + col, t);
          else {
#pragma unroll
            for (int v = 0; v < VEC; ++v) t[v] = 0.0f;
          }
#pragma unroll
          for (int v = 0; v < VEC; ++v) x[u][it * VEC + v] = t[v];
        }
      }
#pragma unroll
      for (int u = 0; u < DEPTH; ++u) {
        if (j0 + u >= cnt) break;
        // batch_access.cpp:118: dest += src * scale
#pragma unroll
        for (int k = 0; k < C; ++k) acc[k] = __fadd_rn(acc[k], __fmul_rn(x[u][k], s[u]));
      }
    }
  }
}

template <int G, int VEC, int ITERS, typename Grp>
__device__ __forceinline__ void reduce_range(const Grp& grp, const PushLaunch& p,
                                             unsigned long long s0, unsigned long long s1,
                                             unsigned D, float (&acc)[VEC * ITERS]) {
#pragma unroll
  for (int k = 0; k < VEC * ITERS; ++k) acc[k] = 0.0f;
  accumulate_global<G, VEC, ITERS>(grp, p, s0, s1, D, acc);
}

// Value held by lane (pos % G) in its register slot pos / G (pos uniform in the group).
template <int PER, typename T, typename Grp>
__device__ __forceinline__ T tile_value(const Grp& grp, const T (&arr)[PER], unsigned pos) {
  constexpr unsigned G = Grp::num_threads();
  const unsigned r = pos / G;
  T v = arr[0];
#pragma unroll
  for (int i = 1; i < PER; ++i) if ((unsigned)i == r) v = arr[i];
  return grp.shfl(v, pos % G);
}

// Accumulates the gradient rows of tile positions [lo, hi) in order, continuing acc.
template <int G, int VEC, int ITERS, int PER, typename Grp>
__device__ __forceinline__ void accumulate_tile(const Grp& grp, const unsigned long long (&gp)[PER],
                                                const float (&sc)[PER], unsigned lo, unsigned hi,
                                                unsigned D, float (&acc)[VEC * ITERS]) {
  constexpr int C = VEC * ITERS;
  constexpr int DEPTH = C <= 4 ? 4 : 2;
  const unsigned gl = grp.thread_rank();
  for (unsigned j0 = lo; j0 < hi; j0 += DEPTH) {
    float x[DEPTH][C];
    float s[DEPTH];
#pragma unroll
    for (int u = 0; u < DEPTH; ++u) {
      const bool use = j0 + u < hi;
      const unsigned pos = use ? j0 + u : lo;
      const unsigned long long q = tile_value<PER>(grp, gp, pos);
      s[u] = tile_value<PER>(grp, sc, pos);
#pragma unroll
      for (int it = 0; it < ITERS; ++it) {
        const unsigned col = (it * G + gl) * VEC;
        float t[VEC];
        if (use && col < D) load_vec<VEC>(reinterpret_cast<const float*>(q) + col, t);
        else {
#pragma unroll
          for (int v = 0; v < VEC; ++v) t[v] = 0.0f;
        }
#pragma unroll
        for (int v = 0; v < VEC; ++v) x[u][it * VEC + v] = t[v];
      }
    }
#pragma unroll
    for (int u = 0; u < DEPTH; ++u) {
      if (j0 + u >= hi) break;
#pragma unroll
      for (int k = 0; k < C; ++k) acc[k] = __fadd_rn(acc[k], __fmul_rn(x[u][k], s[u]));
    }
  }
}

template <int G, int VEC, int ITERS>
__device__ __forceinline__ void load_state(unsigned gl, const float* row, unsigned D,
                                           float (&w)[VEC * ITERS], float (&m)[VEC * ITERS],
                                           float (&v)[VEC * ITERS]) {
#pragma unroll
  for (int it = 0; it < ITERS; ++it) {
    const unsigned col = (it * G + gl) * VEC;
    float a[VEC], b[VEC], c[VEC];
    if (col < D) {
      load_vec<VEC>(row + col, a);
      load_vec<VEC>(row + D + col, b);
      load_vec<VEC>(row + 2 * D + col, c);
    } else {
#pragma unroll
      for (int x = 0; x < VEC; ++x) a[x] = b[x] = c[x] = 0.0f;
    }
#pragma unroll
    for (int x = 0; x < VEC; ++x) { w[it * VEC + x] = a[x]; m[it * VEC + x] = b[x]; v[it * VEC + x] = c[x]; }
  }
}

// LazyAdam on one row (src/update/lazy_adam.cpp:28-37).  Returns reject bits
// (validate) and raises *absmax (apply).
template <int G, int VEC, int ITERS>
__device__ __forceinline__ unsigned adam_row(unsigned gl, const PushTable& T, float* row, unsigned D,
                                             const float (&g)[VEC * ITERS], float (&w)[VEC * ITERS],
                                             float (&m)[VEC * ITERS], float (&v)[VEC * ITERS],
                                             bool apply, bool validate, unsigned* absmax) {
  unsigned bits = 0;
  unsigned mx = 0;
#pragma unroll
  for (int it = 0; it < ITERS; ++it) {
    const unsigned col = (it * G + gl) * VEC;
    if (col >= D) continue;
    float nw[VEC], nm[VEC], nv[VEC];
#pragma unroll
    for (int x = 0; x < VEC; ++x) {
      const int k = it * VEC + x;
      const float gr = g[k];
      const float mm = __fadd_rn(__fmul_rn(T.beta1, m[k]), __fmul_rn(T.one_minus_beta1, gr));
      const float vv = __fadd_rn(__fmul_rn(T.beta2, v[k]),
                                 __fmul_rn(__fmul_rn(T.one_minus_beta2, gr), gr));
      const float ww = __fsub_rn(w[k], __fdiv_rn(__fmul_rn(T.lr_t, mm),
                                                 __fadd_rn(__fsqrt_rn(vv), T.epsilon)));
      if (validate) {
        if (!isfinite(gr)) bits |= kRejectReduction;
        if (!isfinite(mm) || !isfinite(vv) || !isfinite(ww)) bits |= kRejectOptimizer;
      }
      nm[x] = mm; nv[x] = vv;
      nw[x] = clamp_weight(ww, T.has_bounds, T.bound_min, T.bound_max);
      mx = max(mx, max(abs_bits(nw[x]), max(abs_bits(mm), abs_bits(vv))));
    }
    if (apply) {
      store_vec<VEC>(row + col, nw);
      store_vec<VEC>(row + D + col, nm);
      store_vec<VEC>(row + 2 * D + col, nv);
    }
  }
  if (apply) *absmax = max(*absmax, mx);
  return bits;
}

// Run length of key K starting at q (keys sorted), capped at cap+1.
template <int G, typename KeyT, typename Grp>
__device__ __forceinline__ unsigned long long run_forward(const Grp& grp, const void* keys,
                                                          unsigned long long n, unsigned long long q,
                                                          KeyT K, unsigned long long cap) {
  const unsigned gl = grp.thread_rank();
  unsigned long long len = 0;
  while (len <= cap) {
    const unsigned long long i = q + len + gl;
    const bool same = i < n && key_at<KeyT>(keys, i) == K;
    const unsigned ball = grp.ballot(same);
    if (ball != full_mask<G>()) return len + (unsigned long long)(__ffs(~ball) - 1);
    len += G;
  }
  return len;
}

// Number of keys equal to K immediately before position b, capped at cap+1.
template <int G, typename KeyT, typename Grp>
__device__ __forceinline__ unsigned long long run_backward(const Grp& grp, const void* keys,
                                                           unsigned long long b, KeyT K,
                                                           unsigned long long cap) {
  const unsigned gl = grp.thread_rank();
  unsigned long long len = 0;
  while (len <= cap) {
    const bool in = b >= len + gl + 1;
    const bool same = in && key_at<KeyT>(keys, b - len - gl - 1) == K;
    const unsigned ball = grp.ballot(same);
    if (ball != full_mask<G>()) return len + (unsigned long long)(__ffs(~ball) - 1);
    len += G;
  }
  return len;
}

template <int G, int VEC, int ITERS>
__device__ __forceinline__ void store_piece(unsigned gl, float* part, unsigned dim_max,
                                            unsigned long long tile, unsigned D,
                                            const float (&acc)[VEC * ITERS]) {
#pragma unroll
  for (int it = 0; it < ITERS; ++it) {
    const unsigned col = (it * G + gl) * VEC;
    if (col >= D) continue;
    float t[VEC];
#pragma unroll
    for (int x = 0; x < VEC; ++x) t[x] = acc[it * VEC + x];
    store_vec<VEC>(part + tile * dim_max + col, t);
  }
}

// Flush a group's state-bound maximum for table tr (called by all G lanes).
template <typename Grp>
__device__ __forceinline__ void flush_absmax(const Grp& grp, const PushLaunch& p, int tr, unsigned mx) {
  mx = cg::reduce(grp, mx, cg::greater<unsigned>());
  if (grp.thread_rank() == 0 && tr >= 0 && mx) atomicMax(&p.tables[tr].dtable->state_absmax_bits, mx);
}

// ----------------------------------------------------------------- segments
// Shared-memory ring per group: RING slots of [w | m | v | first gradient row].
template <int G, int VEC, int ITERS>
struct SegShape {
  static constexpr int C = VEC * ITERS;
  static constexpr int DCOLS = G * VEC * ITERS;     // columns one group covers
  static constexpr int RING = C <= 4 ? 4 : 2;
  static constexpr int PER = kTile / G;             // tile positions per lane
  static constexpr int GROUPS = 256 / G;
  static constexpr size_t SMEM = (size_t)GROUPS * RING * 4 * DCOLS * sizeof(float);
};

template <int G, int VEC, int ITERS, typename KeyT>
__global__ void __launch_bounds__(256, (VEC * ITERS <= 4) ? 3 : 1) push_segments(PushLaunch p, int pass) {
  const Role R = role(p.control, pass);
  if (!R.run) return;
  using S = SegShape<G, VEC, ITERS>;
  constexpr int C = S::C, DC = S::DCOLS, RING = S::RING, PER = S::PER;
  extern __shared__ float s_ring[];
  const auto grp = cg::tiled_partition<G>(cg::this_thread_block());
  const unsigned gl = grp.thread_rank();
  float* ring = s_ring + (threadIdx.x / G) * (RING * 4 * DC);
  const unsigned long long n = p.n;
  const unsigned long long tiles = (n + kTile - 1) / kTile;
  const unsigned long long gid = (blockIdx.x * (unsigned long long)blockDim.x + threadIdx.x) / G;
  const unsigned long long ngroups = (gridDim.x * (unsigned long long)blockDim.x) / G;
  const KeyT slot_mask = (p.slot_bits >= sizeof(KeyT) * 8) ? ~KeyT(0)
                                                           : ((KeyT(1) << p.slot_bits) - 1);
  const bool work = R.apply || R.validate;
  unsigned bits = 0;
  int cur_tr = -1;
  unsigned cur_max = 0;

  for (unsigned long long t = gid; t < tiles; t += ngroups) {
    const unsigned long long b = t * kTile;
    const unsigned L = (unsigned)min((unsigned long long)kTile, n - b);   // valid positions
    // ---- discovery: keys, segment heads, gradient sources of the whole tile
    KeyT kp[PER];
    unsigned heads = 0;
    KeyT carry = (b > 0) ? key_at<KeyT>(p.keys, b - 1) : KeyT(0);
#pragma unroll
    for (int r = 0; r < PER; ++r) {
      const unsigned j = r * G + gl;
      const bool valid = j < L;
      const KeyT k = valid ? key_at<KeyT>(p.keys, b + j) : KeyT(0);
      KeyT prev = grp.shfl_up(k, 1);
      if (gl == 0) prev = carry;
      const bool head = valid && ((b + j == 0) || k != prev);
      heads |= (unsigned)grp.ballot(head) << (r * G);
      carry = grp.shfl(k, G - 1);
      kp[r] = k;
    }
    unsigned long long gp[PER];
    float sc[PER];
#pragma unroll
    for (int r = 0; r < PER; ++r) {
      const unsigned j = r * G + gl;
      gp[r] = 0;
      sc[r] = 0.0f;
      if (j < L) {
        const unsigned src = __ldg(p.srcs + b + j);
        const unsigned f = src >> kRowBits;
        const unsigned row = src & ((1u << kRowBits) - 1u);
        const PushFeature* F = p.features + f;
        const unsigned Df = __ldg(&F->dim);
        const float* g = reinterpret_cast<const float*>(__ldg(reinterpret_cast<const unsigned long long*>(&F->grad)));
        gp[r] = reinterpret_cast<unsigned long long>(g + (unsigned long long)row * Df);
        sc[r] = __ldg(p.row_scale + __ldg(&F->scale_base) + row);
      }
    }
    const KeyT k_last = tile_value<PER>(grp, kp, L - 1);
    const bool crosses = b + L < n && key_at<KeyT>(p.keys, b + L) == k_last;
    const unsigned first_head = heads ? (unsigned)(__ffs(heads) - 1) : L;
    // ---- a segment that started in an earlier tile
    if (first_head > 0) {
      const KeyT kb = tile_value<PER>(grp, kp, 0);
      const unsigned long long back = run_backward<G, KeyT>(grp, p.keys, b, kb, p.long_run);
      unsigned long long fwd = first_head;
      if (first_head == L && crosses) fwd += run_forward<G, KeyT>(grp, p.keys, n, b + L, kb, p.long_run);
      if (back + fwd > p.long_run && R.partials) {
        const unsigned tr = (unsigned)(kb >> p.slot_bits);
        if (tr < p.table_count) {
          const unsigned D = p.tables[tr].dim;
          float acc[C];
#pragma unroll
          for (int k = 0; k < C; ++k) acc[k] = 0.0f;
          accumulate_tile<G, VEC, ITERS, PER>(grp, gp, sc, 0, first_head, D, acc);
          store_piece<G, VEC, ITERS>(gl, p.part0, p.dim_max, t, D, acc);
        }
      }
    }
    // ---- the last segment starting in the tile may run on (and may be long)
    unsigned short_mask = heads;
    unsigned last_len = 0;
    const int last_start = heads ? 31 - __clz(heads) : -1;
    if (last_start >= 0) {
      last_len = L - (unsigned)last_start;
      unsigned long long tail = 0;
      if (crosses) tail = run_forward<G, KeyT>(grp, p.keys, n, b + L, k_last, p.long_run);
      if ((unsigned long long)last_len + tail > p.long_run) {
        short_mask &= ~(1u << last_start);
        if (R.partials) {
          const unsigned tr = (unsigned)(k_last >> p.slot_bits);
          if (tr < p.table_count) {
            const unsigned D = p.tables[tr].dim;
            float acc[C];
#pragma unroll
            for (int k = 0; k < C; ++k) acc[k] = 0.0f;
            accumulate_tile<G, VEC, ITERS, PER>(grp, gp, sc, (unsigned)last_start, L, D, acc);
            const unsigned which = last_start == 0 ? 0u : 1u;
            store_piece<G, VEC, ITERS>(gl, which ? p.part1 : p.part0, p.dim_max, t, D, acc);
            if (gl == 0) {
              const unsigned at = atomicAdd(&p.control->long_count, 1u);
              p.records[at] = LongRecord{(unsigned long long)k_last, (unsigned)t, which};
            }
          }
        }
      } else {
        last_len = (unsigned)(last_len + tail);
      }
    }
    if (!work || !short_mask) continue;
    // ---- short segments: row state + first gradient row prefetched RING deep
    unsigned issue = short_mask, proc = short_mask;
    const int nseg = __popc(short_mask);
    for (int j = 0; j < nseg + RING - 1; ++j) {
      if (issue) {
        const unsigned s0 = (unsigned)(__ffs(issue) - 1);
        issue &= issue - 1;
        const KeyT K = tile_value<PER>(grp, kp, s0);
        const unsigned tr = (unsigned)(K >> p.slot_bits);
        if (tr < p.table_count) {
          const unsigned D = p.tables[tr].dim;
          const float* row = p.tables[tr].state + (unsigned long long)(K & slot_mask) * 3ull * D;
          const float* g0 = reinterpret_cast<const float*>(tile_value<PER>(grp, gp, s0));
          float* slot = ring + (j % RING) * (4 * DC);
#pragma unroll
          for (int it = 0; it < ITERS; ++it) {
            const unsigned col = (it * G + gl) * VEC;
            if (col < D) {
              cp_async_vec<VEC>(slot + col, row + col);
              cp_async_vec<VEC>(slot + DC + col, row + D + col);
              cp_async_vec<VEC>(slot + 2 * DC + col, row + 2 * D + col);
              cp_async_vec<VEC>(slot + 3 * DC + col, g0 + col);
            }
          }
        }
      }
      cp_async_commit();
      if (j < RING - 1) continue;
      const int jj = j - (RING - 1);
      const unsigned s1 = (unsigned)(__ffs(proc) - 1);
      proc &= proc - 1;
      cp_async_wait<RING - 1>();
      const KeyT K = tile_value<PER>(grp, kp, s1);
      const unsigned tr = (unsigned)(K >> p.slot_bits);
      if (tr >= p.table_count) continue;
      const PushTable& T = p.tables[tr];
      const unsigned D = T.dim;
      // segment length: up to the next head, or last_len for the last one
      const unsigned above = heads & ~((2u << s1) - 1u);
      const unsigned len = above ? (unsigned)(__ffs(above) - 1) - s1 : last_len;
      const unsigned in_tile = min(len, L - s1);
      const float* slot = ring + (jj % RING) * (4 * DC);
      float g[C], w[C], m[C], v[C];
      const float s_first = tile_value<PER>(grp, sc, s1);
#pragma unroll
      for (int it = 0; it < ITERS; ++it) {
        const unsigned col = (it * G + gl) * VEC;
#pragma unroll
        for (int x = 0; x < VEC; ++x) {
          const int k = it * VEC + x;
          const bool in = col + x < D;
          w[k] = in ? slot[col + x] : 0.0f;
          m[k] = in ? slot[DC + col + x] : 0.0f;
          v[k] = in ? slot[2 * DC + col + x] : 0.0f;
          // batch_access.cpp:118: 0 + first term
          g[k] = __fadd_rn(0.0f, __fmul_rn(in ? slot[3 * DC + col + x] : 0.0f, s_first));
        }
      }
      if (in_tile > 1) accumulate_tile<G, VEC, ITERS, PER>(grp, gp, sc, s1 + 1, s1 + in_tile, D, g);
      if (len > in_tile) accumulate_global<G, VEC, ITERS>(grp, p, b + L, b + s1 + len, D, g);
      if ((int)tr != cur_tr) {
        if (R.apply) flush_absmax(grp, p, cur_tr, cur_max);
        cur_tr = (int)tr; cur_max = 0;
      }
      float* grow = T.state + (unsigned long long)(K & slot_mask) * 3ull * D;
      bits |= adam_row<G, VEC, ITERS>(gl, T, grow, D, g, w, m, v, R.apply, R.validate, &cur_max);
      if (R.apply && gl == 0) T.updates[(unsigned long long)(K & slot_mask)] += 1ull;
    }
  }
  bits = cg::reduce(grp, bits, cg::bit_or<unsigned>());
  if (gl == 0 && bits) atomicOr(&p.control->reject_bits, bits);
  if (R.apply) flush_absmax(grp, p, cur_tr, cur_max);
}

// ------------------------------------------------------------ long segments
constexpr int kLongThreads = 512;

template <int G, int VEC, int ITERS, typename KeyT>
__global__ void __launch_bounds__(kLongThreads) push_long(PushLaunch p, int pass) {
  const Role R = role(p.control, pass);
  if (!R.run) return;
  if (!R.apply && !R.validate) return;
  extern __shared__ float s_acc[];   // [groups][dim_max]
  constexpr int C = VEC * ITERS;
  constexpr int NG = kLongThreads / G;
  const auto grp = cg::tiled_partition<G>(cg::this_thread_block());
  const unsigned gl = grp.thread_rank(), w = threadIdx.x / G;
  const unsigned count = *(volatile const unsigned*)&p.control->long_count;
  const unsigned long long n = p.n;
  const unsigned long long tiles = (n + kTile - 1) / kTile;
  const KeyT slot_mask = (p.slot_bits >= sizeof(KeyT) * 8) ? ~KeyT(0)
                                                           : ((KeyT(1) << p.slot_bits) - 1);
  unsigned bits = 0;
  unsigned cur_max = 0;
  int cur_tr = -1;
  for (unsigned rec = blockIdx.x; rec < count; rec += gridDim.x) {
    const LongRecord L = p.records[rec];
    const KeyT K = (KeyT)L.key;
    const unsigned tr = (unsigned)(K >> p.slot_bits);
    const unsigned long long slot = (unsigned long long)(K & slot_mask);
    if (tr >= p.table_count) continue;
    const PushTable& T = p.tables[tr];
    const unsigned D = T.dim;
    // last tile whose first key is K (keys are sorted, so binary search)
    unsigned long long lo = L.first_tile, hi = tiles;   // answer in [lo, hi)
    while (hi - lo > 1) {
      const unsigned long long mid = (lo + hi) >> 1;
      if (key_at<KeyT>(p.keys, mid * kTile) == K) lo = mid; else hi = mid;
    }
    const unsigned long long pieces = lo - L.first_tile + 1;
    // a contiguous chunk of pieces per group, combined afterwards in group order
    const unsigned long long per = (pieces + NG - 1) / NG;
    const unsigned long long p0 = min(pieces, per * w), p1 = min(pieces, p0 + per);
    float acc[C];
#pragma unroll
    for (int k = 0; k < C; ++k) acc[k] = 0.0f;
    for (unsigned long long j0 = p0; j0 < p1; j0 += 4) {
      float x[4][C];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const unsigned long long j = j0 + u;
        const bool use = j < p1;
        const float* src = (j == 0 && L.first_slot) ? p.part1 : p.part0;
        const unsigned long long tile = L.first_tile + j;
#pragma unroll
        for (int it = 0; it < ITERS; ++it) {
          const unsigned col = (it * G + gl) * VEC;
          float t[VEC];
          if (use && col < D) load_vec<VEC>(src + tile * p.dim_max + col, t);
          else {
#pragma unroll
            for (int v = 0; v < VEC; ++v) t[v] = 0.0f;
          }
#pragma unroll
          for (int v = 0; v < VEC; ++v) x[u][it * VEC + v] = t[v];
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (j0 + u >= p1) break;
#pragma unroll
        for (int k = 0; k < C; ++k) acc[k] = __fadd_rn(acc[k], x[u][k]);
      }
    }
#pragma unroll
    for (int it = 0; it < ITERS; ++it) {
      const unsigned col = (it * G + gl) * VEC;
      if (col >= D) continue;
#pragma unroll
      for (int x = 0; x < VEC; ++x) s_acc[w * p.dim_max + col + x] = acc[it * VEC + x];
    }
    __syncthreads();
    if (w == 0) {
      float g[C], wv[C], mv[C], vv[C];
      float* row = T.state + slot * 3ull * D;
      load_state<G, VEC, ITERS>(gl, row, D, wv, mv, vv);
#pragma unroll
      for (int k = 0; k < C; ++k) g[k] = 0.0f;
      for (int x = 0; x < NG; ++x) {
#pragma unroll
        for (int it = 0; it < ITERS; ++it) {
          const unsigned col = (it * G + gl) * VEC;
          if (col >= D) continue;
#pragma unroll
          for (int y = 0; y < VEC; ++y)
            g[it * VEC + y] = __fadd_rn(g[it * VEC + y], s_acc[x * p.dim_max + col + y]);
        }
      }
      if ((int)tr != cur_tr) {
        if (R.apply) flush_absmax(grp, p, cur_tr, cur_max);
        cur_tr = (int)tr; cur_max = 0;
      }
      bits |= adam_row<G, VEC, ITERS>(gl, T, row, D, g, wv, mv, vv, R.apply, R.validate, &cur_max);
      if (R.apply && gl == 0) T.updates[slot] += 1ull;
    }
    __syncthreads();
  }
  if (w == 0) {
    bits = cg::reduce(grp, bits, cg::bit_or<unsigned>());
    if (gl == 0 && bits) atomicOr(&p.control->reject_bits, bits);
    if (R.apply) flush_absmax(grp, p, cur_tr, cur_max);
  }
}

// ----------------------------------------------------------------- finalize
__global__ void push_finalize(PushLaunch p) {
  PushControl* c = p.control;
  const unsigned mode = *(volatile unsigned*)&c->mode;
  const unsigned bits = *(volatile unsigned*)&c->reject_bits;
  const bool accepted = mode != kModeRejected && bits == 0;
  if (accepted) {
    for (unsigned t = threadIdx.x; t < p.table_count; t += blockDim.x) {
      const PushTable& T = p.tables[t];
      DeviceTable* d = T.dtable;
      // src/update/lazy_adam.cpp:39-41
      d->optimizer_sequence += 1ull;
      d->beta1_power = __fmul_rn(d->beta1_power, T.beta1);
      d->beta2_power = __fmul_rn(d->beta2_power, T.beta2);
    }
  }
  if (threadIdx.x == 0) c->accepted = accepted ? 1u : 0u;
}

template <int G, int VEC, int ITERS, typename KeyT>
cudaError_t run_apply(const PushLaunch& p, cudaStream_t s) {
  using SS = SegShape<G, VEC, ITERS>;
  // the shared-memory opt-in is a per-device attribute of the function
  static bool configured[64] = {};
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return e;
  if (device < 0 || device >= 64) return cudaErrorInvalidDevice;
  if (!configured[device]) {
    e = cudaFuncSetAttribute(push_segments<G, VEC, ITERS, KeyT>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SS::SMEM);
    if (e != cudaSuccess) return e;
    configured[device] = true;
  }
  const unsigned long long tiles = (p.n + kTile - 1) / kTile;
  const unsigned long long want = (tiles + SS::GROUPS - 1) / SS::GROUPS;
  const unsigned long long cap = 148ull * ((VEC * ITERS <= 4) ? 3 : 1);
  const unsigned grid = (unsigned)max(1ull, min(want, cap));
  const size_t long_smem = (size_t)(kLongThreads / G) * p.dim_max * sizeof(float);
  const unsigned long_grid = 148 * 2;
  for (int pass = 0; pass < 2; ++pass) {
    if (p.n) push_segments<G, VEC, ITERS, KeyT><<<grid, 256, SS::SMEM, s>>>(p, pass);
    if (p.n) push_long<G, VEC, ITERS, KeyT><<<long_grid, kLongThreads, long_smem, s>>>(p, pass);
  }
  return cudaGetLastError();
}

template <int G, int VEC, int ITERS>
cudaError_t run_key(const PushLaunch& p, cudaStream_t s) {
  return p.key64 ? run_apply<G, VEC, ITERS, unsigned long long>(p, s)
                 : run_apply<G, VEC, ITERS, unsigned int>(p, s);
}
}  // namespace

cudaError_t launch_push_prescan(const PushLaunch& p, cudaStream_t stream) {
  // enough blocks to stream the gradients at full bandwidth
  const unsigned long long per = 256ull * 16;
  const unsigned long long want = (p.grad_values + per - 1) / per;
  const unsigned grid = (unsigned)max(1ull, min(want, 148ull * 8));
  push_prescan<<<grid, 256, 0, stream>>>(p, const_cast<PushTable*>(p.tables));
  return cudaGetLastError();
}

unsigned launch_push_apply_count(const PushLaunch& p) { return p.n ? 4u : 0u; }

cudaError_t launch_push_apply(const PushLaunch& p, cudaStream_t stream) {
  if (p.vec == 4) {
    switch (p.group) {
      case 8: return run_key<8, 4, 1>(p, stream);
      case 16: return run_key<16, 4, 1>(p, stream);
      default:
        if (p.iters == 1) return run_key<32, 4, 1>(p, stream);
        if (p.iters == 2) return run_key<32, 4, 2>(p, stream);
        return run_key<32, 4, 4>(p, stream);
    }
  }
  if (p.iters == 1) return run_key<32, 1, 1>(p, stream);
  if (p.iters == 2) return run_key<32, 1, 2>(p, stream);
  return run_key<32, 1, 4>(p, stream);
}

cudaError_t launch_push_finalize(const PushLaunch& p, cudaStream_t stream) {
  push_finalize<<<1, 32, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace eps_b200
