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
//   prescan    -- finiteness + max|g| of every gradient value (read-only); its
//                 last block computes lr_t per table and picks the mode:
//                 SAFE    when |g_reduced| <= 3*N*max|g| <= 1e17, the recorded
//                         state bound <= 1e17 and lr_t/eps <= 1e20: then no
//                         m, v or w can overflow (|lr_t*m/(sqrt(v)+eps)| <=
//                         1e37) and every row is updated in ONE pass;
//                 CHECKED otherwise: the row kernels validate exactly as the
//                         reference and stage C applies only if nothing was
//                         rejected;
//   pieces     -- push_pieces_uniform (side stream, beside the prescan) for the
//                 uniform shape; stage A sums them itself otherwise;
//   rows       -- push_rows_ring (uniform shape) or push_stage_a;
//   long rows  -- push_stage_b, whose last block advances the beta powers and
//                 the sequence iff the push is accepted (SAFE / REJECTED);
//   stage C    -- the apply pass of a CHECKED push (and its finalize).
//
// Coalescing layout: the occurrences are sorted stably by composite key
// (table rank, slot), the runs of equal keys are compacted into seg_start[U + 1]
// and a row plan (one RowRec per run) is built at lookup time.  A row with one
// occurrence takes 0 + src * scale; a row with 2..64 occurrences gets one piece,
// summed serially in occurrence order (bit-exact with the reference); a longer
// (Zipf-head) row gets ceil(len / 64) pieces, summed in parallel and combined
// in a fixed group tree by one CTA (deterministic; within 1e-6 * sum|terms| of
// the reference's serial sum).
#include <cooperative_groups.h>
#include <cooperative_groups/reduce.h>

#include "kernels.cuh"

namespace cg = cooperative_groups;

#ifndef EPS_PUSH_MIN_BLOCKS
#define EPS_PUSH_MIN_BLOCKS 2         // resident 256-thread blocks per SM of the register
                                      // stages (C <= 4)
#endif
#ifndef EPS_PIECE_DEPTH_REGS
#define EPS_PIECE_DEPTH_REGS 32       // registers per lane for gradient rows in flight
                                      // in the register stage's piece sums
#endif

namespace eps_b200 {
namespace {

template <typename KeyT>
__device__ __forceinline__ KeyT key_at(const void* keys, unsigned long long i) {
  return __ldg(static_cast<const KeyT*>(keys) + i);
}

// ------------------------------------------------------------------ prescan
// The gradient values of every feature, in feature order, form one array of
// grad_values values (grad_prefix[f]: where feature f starts).  Block b scans
// the contiguous span [b * span, (b + 1) * span) of it, feature after feature,
// so the grid's parallelism does not depend on how many features the push has
// (a shard serving 8 requesters x 26 features pushes 208 small tensors).
__global__ void __launch_bounds__(256) push_prescan(PushLaunch p, PushTable* tables_rw) {
  __shared__ unsigned s_bad, s_max, s_last;
  if (threadIdx.x == 0) { s_bad = 0; s_max = 0; }
  __syncthreads();
  const unsigned long long total = p.grad_values;
  const unsigned fc = p.feature_count;
  // a multiple of 4 values: with grad_vec4 every feature starts at one too
  const unsigned long long span = ((total + gridDim.x - 1) / gridDim.x + 3) & ~3ull;
  unsigned long long lo = blockIdx.x * span;
  // a sharded round's requesters reduced every gradient value already
  // (external_reject[1]: their largest |g|): nothing to read here
  const unsigned long long hi = p.external_reject ? lo : min(total, lo + span);
  unsigned bad = 0;
  float mx = 0.0f;
  // the feature holding value `lo`: the last f with grad_prefix[f] <= lo
  unsigned f = 0;
  {
    unsigned a = 0, b = fc;
    while (b - a > 1) { const unsigned m = (a + b) >> 1; if (p.grad_prefix[m] <= lo) a = m; else b = m; }
    f = a;
  }
  for (; lo < hi && f < fc; ++f) {
    const unsigned long long f0 = p.grad_prefix[f], f1 = p.grad_prefix[f + 1];
    const unsigned long long a = max(lo, f0), b = min(hi, f1);
    if (a < b) {
      const float* g = p.features[f].grad + (a - f0);
      if (p.grad_vec4) {
        const float4* g4 = reinterpret_cast<const float4*>(g);
        const unsigned long long n4 = (b - a) / 4;
#pragma unroll 4
        for (unsigned long long i = threadIdx.x; i < n4; i += blockDim.x) {
          const float4 x = __ldg(g4 + i);
          bad |= !isfinite(x.x) | !isfinite(x.y) | !isfinite(x.z) | !isfinite(x.w);
          mx = fmaxf(mx, fmaxf(fmaxf(fabsf(x.x), fabsf(x.y)), fmaxf(fabsf(x.z), fabsf(x.w))));
        }
      } else {
        for (unsigned long long i = threadIdx.x; i < b - a; i += blockDim.x) {
          const float x = __ldg(g + i);
          bad |= !isfinite(x);
          mx = fmaxf(mx, fabsf(x));
        }
      }
    }
    lo = max(lo, b);
  }
  bad = __reduce_or_sync(0xffffffffu, bad);
  unsigned mb = __reduce_max_sync(0xffffffffu, __float_as_uint(mx));
  if (p.external_reject && threadIdx.x == 0) mb = *(volatile const unsigned*)(p.external_reject + 1);
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
  if (*(volatile unsigned*)&c->nonfinite ||
      (p.external_reject && *(volatile const unsigned*)p.external_reject)) {
    c->reject_bits = kRejectNonFiniteInput; c->mode = kModeRejected; return;
  }
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
// Sum of the gradient references [s0, s1) of one coalesced row (all with the
// same key), serially in occurrence order, by the G lanes of `grp` (each lane
// owns VEC*ITERS columns), bit-exact with the reference's serial loop
// g = 0; g += src * scale (src/access/batch_access.cpp:118).  The gradient
// pointers and row-scale bases of the features are staged in shared memory;
// each lane loads its occurrence's row scale together with the rows, the next
// chunk's sources are requested before the current chunk's rows, up to
// DEPTH_REGS / C gradient rows are in flight, and rows past the end add -0.0f
// (the identity).
template <int G, int VEC, int ITERS, int DEPTH_REGS, typename Grp>
__device__ __forceinline__ void reduce_staged(const Grp& grp, const PushLaunch& p,
                                              const float* const* s_grad, const unsigned* s_sbase,
                                              unsigned long long s0, unsigned long long s1,
                                              unsigned D, float (&acc)[VEC * ITERS]) {
  constexpr int C = VEC * ITERS;
  constexpr int DEPTH = G < DEPTH_REGS / C ? G : (DEPTH_REGS / C > 0 ? DEPTH_REGS / C : 1);
  const unsigned gl = grp.thread_rank();
#pragma unroll
  for (int k = 0; k < C; ++k) acc[k] = 0.0f;
  unsigned src = (s0 + gl < s1) ? __ldg(p.srcs + s0 + gl) : 0u;
  for (unsigned long long c0 = s0; c0 < s1; c0 += G) {
    const unsigned long long i = c0 + gl;
    const unsigned f = src >> kRowBits, r = src & ((1u << kRowBits) - 1u);
    const float* rowp = s_grad[f] + (unsigned long long)r * D;
    const float sc = i < s1 ? __ldg(p.row_scale + s_sbase[f] + r) : 0.0f;
    if (i + G < s1) src = __ldg(p.srcs + i + G);
    const int cnt = (int)min((unsigned long long)G, s1 - c0);
#pragma unroll 1
    for (int j0 = 0; j0 < cnt; j0 += DEPTH) {
      float x[DEPTH][C];
      float sv[DEPTH];
#pragma unroll
      for (int u = 0; u < DEPTH; ++u) {
        const float* q = grp.shfl(rowp, (j0 + u) & (G - 1));
        sv[u] = grp.shfl(sc, (j0 + u) & (G - 1));
        const bool use = j0 + u < cnt;
#pragma unroll
        for (int it = 0; it < ITERS; ++it) {
          const unsigned col = (it * G + gl) * VEC;
          float t[VEC];
          if (use && col < D) load_vec<VEC>(q + col, t);
          else {
#pragma unroll
            for (int v = 0; v < VEC; ++v) t[v] = -0.0f;
          }
#pragma unroll
          for (int v = 0; v < VEC; ++v) x[u][it * VEC + v] = t[v];
        }
      }
      // batch_access.cpp:118: dest += src * scale, in occurrence order; the
      // padding rows add (-0) * scale = -0 (scale > 0), the identity
#pragma unroll
      for (int u = 0; u < DEPTH; ++u)
#pragma unroll
        for (int k = 0; k < C; ++k) acc[k] = __fadd_rn(acc[k], __fmul_rn(x[u][k], sv[u]));
    }
  }
}

// Stages every feature's gradient pointer and row-scale base in shared memory.
__device__ __forceinline__ void stage_features(const PushLaunch& p, const float** s_grad,
                                               unsigned* s_sbase) {
  for (unsigned f = threadIdx.x; f < p.feature_count; f += blockDim.x) {
    s_grad[f] = p.features[f].grad;
    s_sbase[f] = (unsigned)p.features[f].scale_base;
  }
  __syncthreads();
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
      store_vec_stream<VEC>(row + col, nw);
      store_vec_stream<VEC>(row + D + col, nm);
      store_vec_stream<VEC>(row + 2 * D + col, nv);
    }
  }
  if (apply) *absmax = max(*absmax, mx);
  return bits;
}

// Flush a group's state-bound maximum for table tr (called by all G lanes).
template <typename Grp>
__device__ __forceinline__ void flush_absmax(const Grp& grp, const PushLaunch& p, int tr, unsigned mx) {
  mx = cg::reduce(grp, mx, cg::greater<unsigned>());
  if (grp.thread_rank() == 0 && tr >= 0 && mx) atomicMax(&p.tables[tr].dtable->state_absmax_bits, mx);
}

template <typename KeyT>
__device__ __forceinline__ KeyT slot_mask_of(unsigned slot_bits) {
  return (slot_bits >= sizeof(KeyT) * 8) ? ~KeyT(0) : ((KeyT(1) << slot_bits) - 1);
}

// ------------------------------------------------------------- row updates
// One coalesced row of the lookup's row plan (rows[u], one 16-byte record per
// run of the sorted keys), updated by a group of G lanes in two steps so that a
// group keeps two rows' loads in flight: `load` issues the gradient-row, [w|m|v]
// and counter loads; `finish` applies LazyAdam and stores.  The gradient is one
// row away: the single occurrence's gradient row times its scale, 0 + src * scale
// (batch_access.cpp:118), or, for a row with 2..long_run occurrences, its piece
// sum reduced in occurrence order in stage A.  The row state is read and
// written with streaming hints (touched once per push).
template <int C>
struct RowRegs {
  float* row;
  const PushTable* T;
  unsigned long long slot, upd;
  unsigned tr;
  bool multi;
  float scale;
  float t[C], w[C], m[C], v[C];
};

template <int G, int VEC, int ITERS, typename KeyT>
__device__ __forceinline__ void load_row(unsigned gl, const PushLaunch& p, const float* const* s_grad,
                                         unsigned long long key, unsigned a, unsigned b, bool apply,
                                         RowRegs<VEC * ITERS>& r) {
  const KeyT K = (KeyT)key;
  r.tr = (unsigned)(K >> p.slot_bits);
  r.T = p.tables + r.tr;
  const unsigned D = r.T->dim;
  r.slot = (unsigned long long)(K & slot_mask_of<KeyT>(p.slot_bits));
  r.row = r.T->state + r.slot * 3ull * D;
  r.multi = (b & kRowMulti) != 0;
  r.scale = r.multi ? 1.0f : __uint_as_float(b);
  const float* q = r.multi ? p.part + (unsigned long long)a * p.dim_max
                           : s_grad[a >> kRowBits] + (unsigned long long)(a & ((1u << kRowBits) - 1u)) * D;
#pragma unroll
  for (int it = 0; it < ITERS; ++it) {
    const unsigned col = (it * G + gl) * VEC;
    float x[VEC], y[VEC], z[VEC], u[VEC];
    if (col < D) {
      load_vec<VEC>(q + col, x);
      load_vec_stream<VEC>(r.row + col, y);
      load_vec_stream<VEC>(r.row + D + col, z);
      load_vec_stream<VEC>(r.row + 2 * D + col, u);
    } else {
#pragma unroll
      for (int k = 0; k < VEC; ++k) x[k] = y[k] = z[k] = u[k] = 0.0f;
    }
#pragma unroll
    for (int k = 0; k < VEC; ++k) {
      r.t[it * VEC + k] = x[k]; r.w[it * VEC + k] = y[k];
      r.m[it * VEC + k] = z[k]; r.v[it * VEC + k] = u[k];
    }
  }
  r.upd = (apply && gl == 0) ? __ldcs(r.T->updates + r.slot) : 0ull;
}

template <int G, int VEC, int ITERS, typename Grp>
__device__ __forceinline__ void finish_row(const Grp& grp, const PushLaunch& p, RowRegs<VEC * ITERS>& r,
                                           bool apply, bool validate, unsigned& bits, int& cur_tr,
                                           unsigned& cur_max) {
  constexpr int C = VEC * ITERS;
  const unsigned gl = grp.thread_rank();
  float g[C];
  if (r.multi) {
#pragma unroll
    for (int k = 0; k < C; ++k) g[k] = r.t[k];
  } else {
    // 0 + src * scale (batch_access.cpp:118)
#pragma unroll
    for (int k = 0; k < C; ++k) g[k] = __fadd_rn(0.0f, __fmul_rn(r.t[k], r.scale));
  }
  if ((int)r.tr != cur_tr) {
    if (apply) flush_absmax(grp, p, cur_tr, cur_max);
    cur_tr = (int)r.tr; cur_max = 0;
  }
  bits |= adam_row<G, VEC, ITERS>(gl, *r.T, r.row, r.T->dim, g, r.w, r.m, r.v, apply, validate, &cur_max);
  if (apply && gl == 0) __stcs(r.T->updates + r.slot, r.upd + 1ull);
}

// Rows [base, base + 32) of the row plan by one warp: one record per lane; the
// warp's groups take the rows round-robin, reading the record fields from the
// owning lane by shuffle.  Software-pipelined: a group issues the loads of its
// next row before it runs LazyAdam on the current one (two register sets,
// ping-pong).  `kinds`: 1 single-occurrence rows, 2 rows with a piece sum,
// 3 both.  Padding and long rows are skipped.
template <int G, int VEC, int ITERS, typename KeyT, typename Grp>
__device__ __forceinline__ void update_chunk(const Grp& grp, const PushLaunch& p,
                                             const float* const* s_grad, unsigned long long base,
                                             unsigned U, unsigned kinds, bool apply, bool validate,
                                             unsigned& bits, int& cur_tr, unsigned& cur_max) {
  constexpr unsigned GPW = 32 / G;
  const unsigned lane = threadIdx.x & 31u, gw = lane / G, gl = grp.thread_rank();
  RowRec rec{0ull, 0u, kRowSkip};
  if (base + lane < U) rec = p.rows[base + lane];
  const unsigned nrow = (unsigned)min(32ull, (unsigned long long)U - base);
  // this group's rows: j = i * GPW + gw for i < iters; a row is used iff its
  // record is of a requested kind (the mask is warp-uniform after the ballots)
  const unsigned kind = rec.b == kRowSkip ? 0u : ((rec.b & kRowMulti) ? 2u : 1u);
  const unsigned mine = __ballot_sync(0xffffffffu, (kind & kinds) != 0 && lane < nrow);
  // lanes j of this group's rows: bit i of `todo` <=> row i * GPW + gw is used
  unsigned todo = 0;
#pragma unroll
  for (unsigned i = 0; i < 32 / GPW; ++i)
    if ((mine >> (i * GPW + gw)) & 1u) todo |= 1u << i;
  RowRegs<VEC * ITERS> r[2];
  // The record fields come from lane jj of the warp; shuffles need every lane
  // of the warp, so all lanes run the same number of steps.
  unsigned cur = todo;
  bool have = false;
  // prime: first used row of this group
  {
    const unsigned i0 = cur ? (unsigned)__ffs(cur) - 1u : 0u;
    const unsigned jj = i0 * GPW + gw;
    const unsigned long long key = __shfl_sync(0xffffffffu, rec.key, jj);
    const unsigned a = __shfl_sync(0xffffffffu, rec.a, jj);
    const unsigned b = __shfl_sync(0xffffffffu, rec.b, jj);
    if (cur) { load_row<G, VEC, ITERS, KeyT>(gl, p, s_grad, key, a, b, apply, r[0]); have = true; cur &= cur - 1u; }
  }
  // every lane runs the same number of steps (shuffles are warp-wide)
  const unsigned steps = __reduce_max_sync(0xffffffffu, (unsigned)__popc(todo));
#pragma unroll 1
  for (unsigned st = 0; st < steps; st += 2) {
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      // issue the next row's loads into r[1 - hh], then finish r[hh]
      const unsigned i1 = cur ? (unsigned)__ffs(cur) - 1u : 0u;
      const unsigned jj = i1 * GPW + gw;
      const unsigned long long key = __shfl_sync(0xffffffffu, rec.key, jj);
      const unsigned a = __shfl_sync(0xffffffffu, rec.a, jj);
      const unsigned b = __shfl_sync(0xffffffffu, rec.b, jj);
      const bool next = cur != 0;
      if (next) { load_row<G, VEC, ITERS, KeyT>(gl, p, s_grad, key, a, b, apply, r[1 - hh]); cur &= cur - 1u; }
      if (have) finish_row<G, VEC, ITERS>(grp, p, r[hh], apply, validate, bits, cur_tr, cur_max);
      have = next;
    }
  }
}

// Gradient of a long row: its pieces [piece_base, piece_base + npieces) summed
// in a fixed tree order -- group x of the block sums the contiguous pieces
// [x * per, (x + 1) * per) in order, then group 0 sums the group partials in
// group order (deterministic; within 1e-6 * sum|terms| of the reference's
// serial sum).  Called by every thread of the block; the result is valid in
// group 0.  s_acc holds (blockDim.x / G) * dim_max floats.
#ifndef EPS_COMBINE_DEPTH
#define EPS_COMBINE_DEPTH 16          // piece sums in flight per group when combining a long row
#endif
constexpr int kCombineDepth = EPS_COMBINE_DEPTH;
template <int G, int VEC, int ITERS, typename Grp>
__device__ __forceinline__ void combine_long(const Grp& grp, const PushLaunch& p, const LongRecord& L,
                                             unsigned D, float* s_acc, float (&g)[VEC * ITERS]) {
  constexpr int C = VEC * ITERS;
  constexpr unsigned NG = 256 / G;
  const unsigned gl = grp.thread_rank(), x = threadIdx.x / G;
  const unsigned per = (L.npieces + NG - 1) / NG;
  const unsigned p0 = min(L.npieces, per * x), p1 = min(L.npieces, p0 + per);
  float acc[C];
#pragma unroll
  for (int k = 0; k < C; ++k) acc[k] = 0.0f;
  for (unsigned j0 = p0; j0 < p1; j0 += kCombineDepth) {
    float r[kCombineDepth][C];
#pragma unroll
    for (int u = 0; u < kCombineDepth; ++u) {
      const bool use = j0 + u < p1;
      const float* q = p.part + ((unsigned long long)L.piece_base + j0 + u) * p.dim_max;
#pragma unroll
      for (int it = 0; it < ITERS; ++it) {
        const unsigned col = (it * G + gl) * VEC;
        float t[VEC];
        if (use && col < D) load_vec<VEC>(q + col, t);
        else {
#pragma unroll
          for (int y = 0; y < VEC; ++y) t[y] = -0.0f;
        }
#pragma unroll
        for (int y = 0; y < VEC; ++y) r[u][it * VEC + y] = t[y];
      }
    }
#pragma unroll
    for (int u = 0; u < kCombineDepth; ++u)
#pragma unroll
      for (int k = 0; k < C; ++k) acc[k] = __fadd_rn(acc[k], r[u][k]);
  }
#pragma unroll
  for (int it = 0; it < ITERS; ++it) {
    const unsigned col = (it * G + gl) * VEC;
    if (col >= D) continue;
#pragma unroll
    for (int y = 0; y < VEC; ++y) s_acc[x * p.dim_max + col + y] = acc[it * VEC + y];
  }
  __syncthreads();
  if (x == 0) {
#pragma unroll
    for (int k = 0; k < C; ++k) g[k] = 0.0f;
    for (unsigned z = 0; z < NG; ++z) {
#pragma unroll
      for (int it = 0; it < ITERS; ++it) {
        const unsigned col = (it * G + gl) * VEC;
        if (col >= D) continue;
#pragma unroll
        for (int y = 0; y < VEC; ++y)
          g[it * VEC + y] = __fadd_rn(g[it * VEC + y], s_acc[z * p.dim_max + col + y]);
      }
    }
  }
}

// Long rows of the plan (one per block at a time): combine, then LazyAdam by
// group 0.  Called by every thread of the block.
template <int G, int VEC, int ITERS, typename KeyT, typename Grp>
__device__ __forceinline__ void update_long_rows(const Grp& grp, const PushLaunch& p, float* s_acc,
                                                 unsigned* counter, bool apply, bool validate,
                                                 unsigned& bits, int& cur_tr, unsigned& cur_max) {
  constexpr int C = VEC * ITERS;
  __shared__ unsigned s_rec;
  const unsigned gl = grp.thread_rank();
  const unsigned count = *(volatile const unsigned*)&p.plan->long_count;
  const KeyT smask = slot_mask_of<KeyT>(p.slot_bits);
  // records are claimed per block from `counter` (or taken grid-stride without one)
  auto next = [&](unsigned prev) -> unsigned {
    if (!counter) return prev + gridDim.x;
    __syncthreads();                       // every thread has read s_rec
    if (threadIdx.x == 0) s_rec = atomicAdd(counter, 1u);
    __syncthreads();
    return s_rec;
  };
  for (unsigned rec = counter ? next(0) : blockIdx.x; rec < count; rec = next(rec)) {
    const LongRecord L = p.records[rec];
    const KeyT K = (KeyT)L.key;
    const unsigned tr = (unsigned)(K >> p.slot_bits);
    const PushTable& T = p.tables[tr];
    const unsigned D = T.dim;
    float g[C];
    combine_long<G, VEC, ITERS>(grp, p, L, D, s_acc, g);
    if (threadIdx.x < G) {
      const unsigned long long slot = (unsigned long long)(K & smask);
      float* row = T.state + slot * 3ull * D;
      float w[C], m[C], v[C];
      load_state<G, VEC, ITERS>(gl, row, D, w, m, v);
      if ((int)tr != cur_tr) {
        if (apply) flush_absmax(grp, p, cur_tr, cur_max);
        cur_tr = (int)tr; cur_max = 0;
      }
      bits |= adam_row<G, VEC, ITERS>(gl, T, row, D, g, w, m, v, apply, validate, &cur_max);
      if (apply && gl == 0) T.updates[slot] += 1ull;
    }
    __syncthreads();                       // s_acc is reused
  }
}

// Flush a block's reject bits and state bound; then the last block of the
// launch (counted in *done) runs `last` once every other block's writes are
// visible.  Called by every thread of the block.
template <typename Grp>
__device__ __forceinline__ bool flush_and_count(const Grp& grp, const PushLaunch& p, unsigned bits,
                                                bool apply, int cur_tr, unsigned cur_max,
                                                unsigned* done) {
  __shared__ unsigned s_last;
  bits = cg::reduce(grp, bits, cg::bit_or<unsigned>());
  if (grp.thread_rank() == 0 && bits) atomicOr(&p.control->reject_bits, bits);
  if (apply) flush_absmax(grp, p, cur_tr, cur_max);
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(done, 1u) == gridDim.x - 1;
  __syncthreads();
  if (s_last) __threadfence();
  return s_last;
}

// src/update/lazy_adam.cpp:39-41: once per table iff the push is accepted.
__device__ __forceinline__ void finalize_tables(const PushLaunch& p) {
  PushControl* c = p.control;
  const unsigned mode = *(volatile unsigned*)&c->mode;
  const unsigned bits = *(volatile unsigned*)&c->reject_bits;
  const bool accepted = mode != kModeRejected && bits == 0;
  if (accepted) {
    for (unsigned t = threadIdx.x; t < p.table_count; t += blockDim.x) {
      const PushTable& T = p.tables[t];
      DeviceTable* d = T.dtable;
      d->optimizer_sequence += 1ull;
      d->beta1_power = __fmul_rn(d->beta1_power, T.beta1);
      d->beta2_power = __fmul_rn(d->beta2_power, T.beta2);
    }
  }
  if (threadIdx.x == 0) c->accepted = accepted ? 1u : 0u;
}

// ----------------------------------------------------------------- stage A
// Piece sums and single-occurrence rows in one launch, interleaved so that the
// L2-bound piece reductions (gradient rows re-read per occurrence) overlap the
// HBM-bound read-modify-write of single rows: the launch's chunk sequence
// holds R row chunks (32 plan records) and Q piece chunks (kChunkPieces pieces
// per group), chunk c being a piece chunk iff floor((c+1)Q/T) > floor(cQ/T)
// (T = R + Q); warps take chunks grid-stride.  SAFE mode applies single rows
// here; CHECKED mode only validates them (stage C applies).
constexpr unsigned kChunkPieces = 1;
template <int G, int VEC, int ITERS, typename KeyT>
__global__ void __launch_bounds__(256, (VEC * ITERS <= 4) ? EPS_PUSH_MIN_BLOCKS : 2) push_stage_a(PushLaunch p) {
  __shared__ const float* s_grad[kMaxFeatures];
  __shared__ unsigned s_sbase[kMaxFeatures];
  const unsigned mode = *(volatile const unsigned*)&p.control->mode;
  if (mode == kModeRejected) return;
  const bool apply = mode == kModeSafe, validate = mode == kModeChecked;
  stage_features(p, s_grad, s_sbase);
  constexpr int C = VEC * ITERS;
  constexpr unsigned GPW = 32 / G;
  const auto grp = cg::tiled_partition<G>(cg::this_thread_block());
  const unsigned gl = grp.thread_rank();
  const unsigned lane = threadIdx.x & 31u, gw = lane / G;
  const unsigned U = *(volatile const unsigned*)p.seg_total;
  const unsigned P = *(volatile const unsigned*)&p.plan->piece_count;
  // with the ring path (push_rows_ring) this launch reduces only the pieces
  const unsigned long long R = p.ring_dim ? 0ull : (U + 31ull) / 32ull;
  const unsigned long long Q = (P + kChunkPieces * GPW - 1ull) / (kChunkPieces * GPW);
  const unsigned long long T = R + Q;
  unsigned bits = 0;
  int cur_tr = -1;
  unsigned cur_max = 0;
  // chunks are claimed dynamically (one counter per launch); the next claim is
  // issued before the current chunk is processed
  unsigned claim = 0;
  if (lane == 0) claim = atomicAdd(&p.control->work_a, 1u);
  unsigned long long c = __shfl_sync(0xffffffffu, claim, 0);
  while (c < T) {
    if (lane == 0) claim = atomicAdd(&p.control->work_a, 1u);
    const unsigned long long qb = c * Q / T, qa = (c + 1) * Q / T;
    if (qa > qb) {
      for (unsigned k = 0; k < kChunkPieces; ++k) {
        const unsigned long long item = (qb * GPW + gw) * kChunkPieces + k;
        if (item >= P) break;
        const uint2 pc = p.pieces[item];
        const KeyT K = key_at<KeyT>(p.keys, pc.x);
        const unsigned D = p.tables[(unsigned)(K >> p.slot_bits)].dim;
        float acc[C];
        reduce_staged<G, VEC, ITERS, EPS_PIECE_DEPTH_REGS>(grp, p, s_grad, s_sbase, pc.x,
                                                           (unsigned long long)pc.x + pc.y, D, acc);
#pragma unroll
        for (int it = 0; it < ITERS; ++it) {
          const unsigned col = (it * G + gl) * VEC;
          if (col >= D) continue;
          float t[VEC];
#pragma unroll
          for (int x = 0; x < VEC; ++x) t[x] = acc[it * VEC + x];
          store_vec<VEC>(p.part + item * p.dim_max + col, t);
        }
      }
    } else {
      update_chunk<G, VEC, ITERS, KeyT>(grp, p, s_grad, (c - qb) * 32ull, U, 1u, apply, validate,
                                        bits, cur_tr, cur_max);
    }
    c = __shfl_sync(0xffffffffu, claim, 0);
  }
  bits = cg::reduce(grp, bits, cg::bit_or<unsigned>());
  if (gl == 0 && bits) atomicOr(&p.control->reject_bits, bits);
  if (apply) flush_absmax(grp, p, cur_tr, cur_max);
}

// ----------------------------------------------- pieces for the uniform shape
// The piece sums of stage A for the common shape (every table has dimension D
// in {32, 64, 128}): a group of G = D / 4 lanes reduces one piece at a time,
// serially in occurrence order (reduce_staged's arithmetic), with the latency
// of the index loads taken off the chain: pieces are claimed one at a time
// (the descriptor of the next claim loaded a claim ahead; claiming several
// contiguous long-row pieces at once left a tail: cfg2 68 -> 45 us), and the
// first sources of the next piece are loaded while the current piece is summed.
#ifndef EPS_PIECES_DEPTH
#define EPS_PIECES_DEPTH 8            // gradient rows in flight per group
#endif
#ifndef EPS_PIECES_MIN_BLOCKS
#define EPS_PIECES_MIN_BLOCKS 3
#endif
#ifndef EPS_PIECES_PER_CLAIM
#define EPS_PIECES_PER_CLAIM 1        // long-row pieces are contiguous: claim them singly
#endif
constexpr unsigned kPiecesPerClaim = EPS_PIECES_PER_CLAIM;
template <int D>
__global__ void __launch_bounds__(256, EPS_PIECES_MIN_BLOCKS) push_pieces_uniform(PushLaunch p) {
  constexpr int G = D / 4;
  constexpr int DEPTH = EPS_PIECES_DEPTH;
  __shared__ const float* s_grad[kMaxFeatures];
  __shared__ unsigned s_sbase[kMaxFeatures];
  // runs concurrently with the prescan (it writes no state, so the push's
  // accept/reject decision is not needed); an invalid lookup's plan may hold
  // sources its occurrence list never wrote, so nothing is summed then
  if (*(volatile const unsigned*)p.lookup_error) return;
  stage_features(p, s_grad, s_sbase);
  const auto grp = cg::tiled_partition<G>(cg::this_thread_block());
  const unsigned gl = grp.thread_rank();
  const unsigned P = *(volatile const unsigned*)&p.plan->piece_count;
  auto claim = [&]() -> unsigned {
    unsigned c = 0;
    if (gl == 0) c = atomicAdd(&p.control->work_a, kPiecesPerClaim);
    return grp.shfl(c, 0);
  };
  auto descs = [&](unsigned b) -> uint2 {
    return (gl < kPiecesPerClaim && b + gl < P) ? p.pieces[b + gl] : make_uint2(0u, 0u);
  };
  auto first_src = [&](uint2 pc) -> unsigned { return gl < pc.y ? __ldg(p.srcs + pc.x + gl) : 0u; };
  unsigned base = claim();
  uint2 pcs = descs(base);
  unsigned nbase = claim();
  uint2 npcs = descs(nbase);
  unsigned src = first_src(make_uint2(grp.shfl(pcs.x, 0), grp.shfl(pcs.y, 0)));
  while (base < P) {
#pragma unroll 1
    for (unsigned k = 0; k < kPiecesPerClaim && base + k < P; ++k) {
      const uint2 pc = make_uint2(grp.shfl(pcs.x, k), grp.shfl(pcs.y, k));
      // the next piece's first sources, in flight during this piece
      const bool last_here = k + 1 == kPiecesPerClaim || base + k + 1 >= P;
      const uint2 pn = last_here ? make_uint2(grp.shfl(npcs.x, 0), grp.shfl(npcs.y, 0))
                                 : make_uint2(grp.shfl(pcs.x, k + 1), grp.shfl(pcs.y, k + 1));
      const bool has_next = last_here ? nbase < P : true;
      const unsigned nsrc = has_next ? first_src(pn) : 0u;
      float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      for (unsigned c0 = 0; c0 < pc.y; c0 += G) {
        const unsigned f = src >> kRowBits, r = src & ((1u << kRowBits) - 1u);
        const float* rowp = s_grad[f] + (unsigned long long)r * D;
        const float sc = c0 + gl < pc.y ? __ldg(p.row_scale + s_sbase[f] + r) : 0.0f;
        if (c0 + G + gl < pc.y) src = __ldg(p.srcs + pc.x + c0 + G + gl);
        const int cnt = (int)min((unsigned)G, pc.y - c0);
#pragma unroll 1
        for (int j0 = 0; j0 < cnt; j0 += DEPTH) {
          float x[DEPTH][4];
          float sv[DEPTH];
#pragma unroll
          for (int u = 0; u < DEPTH; ++u) {
            const float* q = grp.shfl(rowp, (j0 + u) & (G - 1));
            sv[u] = grp.shfl(sc, (j0 + u) & (G - 1));
            if (j0 + u < cnt) {
              const float4 t = *reinterpret_cast<const float4*>(q + 4 * gl);
              x[u][0] = t.x; x[u][1] = t.y; x[u][2] = t.z; x[u][3] = t.w;
            } else {
              x[u][0] = x[u][1] = x[u][2] = x[u][3] = -0.0f;
            }
          }
          // dest += src * scale in occurrence order (batch_access.cpp:118)
#pragma unroll
          for (int u = 0; u < DEPTH; ++u)
#pragma unroll
            for (int v = 0; v < 4; ++v) acc[v] = __fadd_rn(acc[v], __fmul_rn(x[u][v], sv[u]));
        }
      }
      *reinterpret_cast<float4*>(p.part + (unsigned long long)(base + k) * D + 4 * gl) =
          make_float4(acc[0], acc[1], acc[2], acc[3]);
      src = nsrc;
    }
    base = nbase;
    pcs = npcs;
    if (base < P) {
      nbase = claim();
      npcs = descs(nbase);
    }
  }
}

template <int D>
cudaError_t run_pieces_uniform(const PushLaunch& p, cudaStream_t s) {
  const unsigned long long want = (p.n / 2 + 255) / 256;
  const unsigned grid = (unsigned)max(1ull, min(want, 148ull * EPS_PIECES_MIN_BLOCKS));
  push_pieces_uniform<D><<<grid, 256, 0, s>>>(p);
  return cudaGetLastError();
}

// --------------------------------------------------- rows through an async ring
// The row updates for the common shape (every table of the push has the same
// dimension D in {32, 64, 128}; 16-byte aligned gradients).  A warp works in
// steps of 32 / G rows, one per group of G = D / 4 lanes (one float4 of each of
// w, m, v and g per lane), and keeps the rows of the next kRingSlots / (32 / G)
// - 1 steps in flight through a ring of shared-memory slots filled by cp.async
// (16-byte per-lane asynchronous copies, one commit group per step): the
// [w|m|v] row, the row's gradient (the single occurrence's gradient row or,
// for 2..long_run occurrences, its in-order piece sum) and the 16-byte block
// holding its counter.  Rows in flight hold no registers, so an SM keeps
// warps x kRingSlots rows in flight.  Rows come from chunks of 32 plan records
// claimed dynamically; the next chunk's records load while the current chunk is
// issued.  Long rows and padding rows are skipped (stage B).
constexpr int kRingSlots = 8;
constexpr unsigned long long kEmptySlot = ~0ull;
template <int D> struct RingShape {
  static constexpr int kGroup = D / 4;                    // lanes per row
  static constexpr int kRows = 32 / kGroup;               // rows per step
  static constexpr int kSteps = kRingSlots / kRows;       // steps in the ring
  static constexpr int kSlot = 4 * D + 8;                 // floats: w, m, v, g, counter block, key
  static constexpr int kWarps = D >= 128 ? 4 : 8;          // warps per block
  static constexpr size_t kBytes = (size_t)kWarps * kRingSlots * kSlot * sizeof(float);
};  // D = 64: 67.6 KB ring + 3.6 KB descriptors per block, three blocks per SM

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit_group() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }

// LazyAdam parameters of one table, held in registers while a warp's rows
// stay in that table.
struct AdamRegs {
  float b1, o1, b2, o2, lr, eps, lo, hi;
  int bounded;
  float* state;
  unsigned long long* updates;
};
__device__ __forceinline__ AdamRegs adam_regs(const PushTable& T) {
  return AdamRegs{T.beta1, T.one_minus_beta1, T.beta2, T.one_minus_beta2, T.lr_t, T.epsilon,
                  T.bound_min, T.bound_max, T.has_bounds, T.state, T.updates};
}

// LazyAdam on N consecutive elements of one row (src/update/lazy_adam.cpp:28-37),
// in place; VALIDATE returns the reject bits, APPLY raises *mx to the largest
// |w|, |m|, v written.
template <int N, bool APPLY, bool VALIDATE>
__device__ __forceinline__ unsigned adam_elems(const AdamRegs& P, const float (&g)[N], float (&w)[N],
                                               float (&m)[N], float (&v)[N], float& mx) {
  unsigned bits = 0;
#pragma unroll
  for (int x = 0; x < N; ++x) {
    const float mm = __fadd_rn(__fmul_rn(P.b1, m[x]), __fmul_rn(P.o1, g[x]));
    const float vv = __fadd_rn(__fmul_rn(P.b2, v[x]), __fmul_rn(__fmul_rn(P.o2, g[x]), g[x]));
    const float ww = __fsub_rn(w[x], __fdiv_rn(__fmul_rn(P.lr, mm), __fadd_rn(__fsqrt_rn(vv), P.eps)));
    if (VALIDATE) {
      if (!isfinite(g[x])) bits |= kRejectReduction;
      if (!isfinite(mm) || !isfinite(vv) || !isfinite(ww)) bits |= kRejectOptimizer;
    }
    m[x] = mm; v[x] = vv; w[x] = ww;
  }
  if (P.bounded) {
#pragma unroll
    for (int x = 0; x < N; ++x) w[x] = w[x] < P.lo ? P.lo : (P.hi < w[x] ? P.hi : w[x]);
  }
  if (APPLY) {
#pragma unroll
    for (int x = 0; x < N; ++x) mx = fmaxf(mx, fmaxf(fabsf(w[x]), fmaxf(fabsf(m[x]), fabsf(v[x]))));
  }
  return bits;
}

template <int D, typename KeyT, bool APPLY, bool VALIDATE>
__device__ __forceinline__ void ring_rows(const PushLaunch& p, const PushTable* s_tab, bool tabs_shared,
                                          const float* const* s_feat, bool feats_shared) {
  using S = RingShape<D>;
  constexpr int G = S::kGroup, RP = S::kRows, NS = S::kSteps;
  extern __shared__ float4 ring_smem[];
  const auto grp = cg::tiled_partition<G>(cg::this_thread_block());
  const unsigned lane = threadIdx.x & 31u, gw = lane / G, gl = grp.thread_rank();
  float* const ring = reinterpret_cast<float*>(ring_smem) + (threadIdx.x >> 5) * (kRingSlots * S::kSlot);
  const unsigned U = *(volatile const unsigned*)p.seg_total;
  const unsigned long long R = (U + 31ull) / 32ull;
  const unsigned slot_bits = p.slot_bits;
  const KeyT smask = slot_mask_of<KeyT>(slot_bits);
  auto table = [&](unsigned tr) -> const PushTable& { return tabs_shared ? s_tab[tr] : p.tables[tr]; };

  // ---- producer: the chunk being issued (records one per lane, mask of the
  // rows still to issue) and the next chunk (records loaded ahead)
  auto claim_chunk = [&]() -> unsigned long long {
    unsigned c = 0;
    if (lane == 0) c = atomicAdd(&p.control->work_ring, 1u);
    return __shfl_sync(0xffffffffu, c, 0);
  };
  auto load_chunk = [&](unsigned long long c, RowRec& rec) {
    rec = RowRec{0ull, 0u, kRowSkip};
    if (c < R && c * 32ull + lane < U) rec = p.rows[c * 32ull + lane];
  };
  unsigned long long c_cur = claim_chunk();
  RowRec r_cur, r_nxt;
  load_chunk(c_cur, r_cur);
  unsigned long long c_nxt = c_cur < R ? claim_chunk() : R;
  load_chunk(c_nxt, r_nxt);
  bool more = c_cur < R;
  unsigned m_cur = __ballot_sync(0xffffffffu, r_cur.b != kRowSkip);
  int p_tr = -1;                          // producer's cached table
  const float* p_state = nullptr;
  const unsigned long long* p_upd = nullptr;

  // issues the next step's rows into the step's slots, all groups at once:
  // group h takes the h-th remaining row of the current chunk (a step never
  // spans two chunks; groups without a row write an empty marker); one commit
  // group per call; returns whether any row was issued
  auto produce = [&](int step) -> bool {
    while (more && m_cur == 0) {
      c_cur = c_nxt; r_cur = r_nxt;
      more = c_cur < R;
      if (!more) break;
      m_cur = __ballot_sync(0xffffffffu, r_cur.b != kRowSkip);
      c_nxt = claim_chunk();
      load_chunk(c_nxt, r_nxt);
    }
    unsigned mine = more ? m_cur : 0u;
#pragma unroll
    for (int h = 0; h < RP - 1; ++h)
      if ((unsigned)h < gw) mine &= mine - 1u;
    const bool has = mine != 0;
    const int j = has ? __ffs(mine) - 1 : 0;
#pragma unroll
    for (int h = 0; h < RP; ++h) m_cur &= m_cur - 1u;
    const unsigned long long key = __shfl_sync(0xffffffffu, r_cur.key, j);
    const unsigned a = __shfl_sync(0xffffffffu, r_cur.a, j);
    const unsigned b = __shfl_sync(0xffffffffu, r_cur.b, j);
    float* slot = ring + (step * RP + gw) * S::kSlot;
    if (has) {
      const KeyT K = (KeyT)key;
      const int tr = (int)(K >> slot_bits);
      if (tr != p_tr) { const PushTable& T = table((unsigned)tr); p_state = T.state; p_upd = T.updates; p_tr = tr; }
      const unsigned long long sl = (unsigned long long)(K & smask);
      const float* st = p_state + sl * (3ull * D);
      const unsigned f = a >> kRowBits;
      const float* gr = (b & kRowMulti) ? p.part + (unsigned long long)a * D
                                        : (feats_shared ? s_feat[f] : p.features[f].grad) +
                                              (unsigned long long)(a & ((1u << kRowBits) - 1u)) * D;
      // [w|m|v]: 3G 16-byte pieces, three per lane; gradient: one per lane
#pragma unroll
      for (int q = 0; q < 3; ++q) cp_async16(slot + 4 * (q * G + gl), st + 4 * (q * G + gl));
      cp_async16(slot + 3 * D + 4 * gl, gr + 4 * gl);
      if (gl == 0) cp_async16(slot + 4 * D, p_upd + (sl & ~1ull));
    }
    if (gl == 0) {
      *reinterpret_cast<unsigned long long*>(slot + 4 * D + 4) = has ? key : kEmptySlot;
      // a single row's gradient is its occurrence's row times the row scale;
      // a piece sum is used as summed (times 1, exact)
      slot[4 * D + 6] = (b & kRowMulti) ? 1.0f : __uint_as_float(b);
    }
    cp_async_commit_group();
    return __any_sync(0xffffffffu, has);
  };

  unsigned bits = 0;
  int cur_tr = -1;
  float cur_max = 0.0f;
  AdamRegs P{};
  int live = 0;                          // steps in the ring holding rows
#pragma unroll
  for (int k = 0; k < NS - 1; ++k) live += produce(k) ? 1 : 0;
  // step t: issue into ring step (t - 1) % NS (consumed at t - 1), then consume
  // ring step t % NS; unrolled over the ring so that slot offsets are constants
  bool done = live == 0 && !more;
  while (!done) {
#pragma unroll
    for (int k = 0; k < NS; ++k) {
      live += produce((k + NS - 1) % NS) ? 1 : 0;
      asm volatile("cp.async.wait_group %0;\n" ::"n"(NS - 1) : "memory");
      __syncwarp();
      const float* s = ring + (k * RP + gw) * S::kSlot;
      const unsigned long long key = *reinterpret_cast<const unsigned long long*>(s + 4 * D + 4);
      const bool step_used = __any_sync(0xffffffffu, key != kEmptySlot);
      if (key != kEmptySlot) {
        const KeyT K = (KeyT)key;
        const int tr = (int)(K >> slot_bits);
        if (tr != cur_tr) {
          if (APPLY) flush_absmax(grp, p, cur_tr, __float_as_uint(cur_max));
          P = adam_regs(table((unsigned)tr));
          cur_tr = tr; cur_max = 0.0f;
        }
        const unsigned long long sl = (unsigned long long)(K & smask);
        float w[4], m[4], v[4], g[4];
        load_vec<4>(s + 4 * gl, w);
        load_vec<4>(s + D + 4 * gl, m);
        load_vec<4>(s + 2 * D + 4 * gl, v);
        load_vec<4>(s + 3 * D + 4 * gl, g);
        // 0 + src * scale for a single row (batch_access.cpp:118); a piece sum
        // (scale 1) starts from +0 and is never -0, so 0 + sum * 1 leaves it unchanged
        const float scale = s[4 * D + 6];
#pragma unroll
        for (int x = 0; x < 4; ++x) g[x] = __fadd_rn(0.0f, __fmul_rn(g[x], scale));
        bits |= adam_elems<4, APPLY, VALIDATE>(P, g, w, m, v, cur_max);
        if (APPLY) {
          float* row = P.state + sl * (3ull * D) + 4 * gl;
          store_vec_stream<4>(row, w);
          store_vec_stream<4>(row + D, m);
          store_vec_stream<4>(row + 2 * D, v);
          if (gl == 0) {
            const unsigned long long upd = *reinterpret_cast<const unsigned long long*>(s + 4 * D + 2 * (sl & 1ull));
            __stcs(P.updates + sl, upd + 1ull);
          }
        }
      }
      live -= step_used ? 1 : 0;
      __syncwarp();
      if (live == 0 && !more) { done = true; break; }
    }
  }
  asm volatile("cp.async.wait_group 0;\n" ::: "memory");
  bits = cg::reduce(grp, bits, cg::bit_or<unsigned>());
  if (gl == 0 && bits) atomicOr(&p.control->reject_bits, bits);
  if (APPLY) flush_absmax(grp, p, cur_tr, __float_as_uint(cur_max));
}

template <int D, typename KeyT>
__global__ void __launch_bounds__(RingShape<D>::kWarps * 32) push_rows_ring(PushLaunch p) {
  // table and feature descriptors of small pushes live in shared memory: the
  // large ring leaves little L1, and a descriptor miss would stall the warp
  constexpr unsigned kTabs = 32, kFeats = 128;
  __shared__ PushTable s_tab[kTabs];
  __shared__ const float* s_feat[kFeats];
  const unsigned mode = *(volatile const unsigned*)&p.control->mode;
  if (mode == kModeRejected) return;
  for (unsigned i = threadIdx.x; i < min(p.table_count, kTabs); i += blockDim.x) s_tab[i] = p.tables[i];
  for (unsigned i = threadIdx.x; i < min(p.feature_count, kFeats); i += blockDim.x) s_feat[i] = p.features[i].grad;
  __syncthreads();
  const bool tabs_shared = p.table_count <= kTabs, feats_shared = p.feature_count <= kFeats;
  if (mode == kModeSafe) ring_rows<D, KeyT, true, false>(p, s_tab, tabs_shared, s_feat, feats_shared);
  else ring_rows<D, KeyT, false, true>(p, s_tab, tabs_shared, s_feat, feats_shared);
}

// ----------------------------------------------------------------- stage B
// Long rows (block-level combine of their pieces) and rows with a piece sum;
// SAFE mode applies, CHECKED mode validates.  Unless the push is CHECKED, the
// launch's last block then advances the beta powers iff it was accepted.
template <int G, int VEC, int ITERS, typename KeyT>
__global__ void __launch_bounds__(256, (VEC * ITERS <= 4) ? EPS_PUSH_MIN_BLOCKS : 2) push_stage_b(PushLaunch p) {
  __shared__ const float* s_grad[kMaxFeatures];
  __shared__ unsigned s_sbase[kMaxFeatures];
  extern __shared__ float s_acc[];
  const unsigned mode = *(volatile const unsigned*)&p.control->mode;
  const auto grp = cg::tiled_partition<G>(cg::this_thread_block());
  if (mode == kModeRejected) {
    if (blockIdx.x == 0) finalize_tables(p);
    return;
  }
  const bool apply = mode == kModeSafe, validate = mode == kModeChecked;
  stage_features(p, s_grad, s_sbase);
  unsigned bits = 0;
  int cur_tr = -1;
  unsigned cur_max = 0;
  update_long_rows<G, VEC, ITERS, KeyT>(grp, p, s_acc, &p.control->work_long, apply, validate, bits,
                                        cur_tr, cur_max);
  const unsigned U = *(volatile const unsigned*)p.seg_total;
  const unsigned lane = threadIdx.x & 31u;
  unsigned claim = 0;
  if (lane == 0) claim = atomicAdd(&p.control->work_b, 1u);
  unsigned long long c = __shfl_sync(0xffffffffu, claim, 0);
  while (!p.ring_dim && c * 32ull < U) {
    if (lane == 0) claim = atomicAdd(&p.control->work_b, 1u);
    update_chunk<G, VEC, ITERS, KeyT>(grp, p, s_grad, c * 32ull, U, 2u, apply, validate, bits,
                                      cur_tr, cur_max);
    c = __shfl_sync(0xffffffffu, claim, 0);
  }
  if (flush_and_count(grp, p, bits, apply, cur_tr, cur_max, &p.control->blocks_done_b) &&
      mode != kModeChecked)
    finalize_tables(p);
}

// ----------------------------------------------------------------- stage C
// CHECKED mode only: when stages A and B rejected nothing, apply every row
// (recomputing the same gradients), then the last block finalizes.
template <int G, int VEC, int ITERS, typename KeyT>
__global__ void __launch_bounds__(256, (VEC * ITERS <= 4) ? EPS_PUSH_MIN_BLOCKS : 2) push_stage_c(PushLaunch p) {
  __shared__ const float* s_grad[kMaxFeatures];
  __shared__ unsigned s_sbase[kMaxFeatures];
  extern __shared__ float s_acc[];
  const unsigned mode = *(volatile const unsigned*)&p.control->mode;
  if (mode != kModeChecked) return;
  const auto grp = cg::tiled_partition<G>(cg::this_thread_block());
  const bool apply = *(volatile const unsigned*)&p.control->reject_bits == 0;
  unsigned bits = 0;
  int cur_tr = -1;
  unsigned cur_max = 0;
  if (apply) {
    stage_features(p, s_grad, s_sbase);
    update_long_rows<G, VEC, ITERS, KeyT>(grp, p, s_acc, nullptr, true, false, bits, cur_tr, cur_max);
    const unsigned U = *(volatile const unsigned*)p.seg_total;
    const unsigned long long warp = (blockIdx.x * (unsigned long long)blockDim.x + threadIdx.x) >> 5;
    const unsigned long long nwarps = (gridDim.x * (unsigned long long)blockDim.x) >> 5;
    for (unsigned long long c = warp; c * 32ull < U; c += nwarps)
      update_chunk<G, VEC, ITERS, KeyT>(grp, p, s_grad, c * 32ull, U, 3u, true, false, bits,
                                        cur_tr, cur_max);
  }
  if (flush_and_count(grp, p, 0u, apply, cur_tr, cur_max, &p.control->blocks_done_c))
    finalize_tables(p);
}
// --------------------------------------------------- agent-style updates
// CacheBackend::ApplyHost (src/cache/host_backend.cpp:119-146): LazyAdam with the
// caller's optimizer context on unique rows, all-or-nothing, no power advance.
// With `compact`, each row's gradient is first expanded from the CSR references
// in order (ExpandCompactGradients, src/access/compact_gradients.cpp:27-39:
// sum = 0; sum += source * scale).  Pass 0 validates, pass 1 applies iff pass 0
// rejected nothing.
template <int G, int VEC, int ITERS>
__global__ void __launch_bounds__(256) apply_rows_kernel(ApplyLaunch p, int pass) {
  if (pass == 1 && *(volatile const unsigned*)p.reject) return;
  constexpr int C = VEC * ITERS;
  const auto grp = cg::tiled_partition<G>(cg::this_thread_block());
  const unsigned gl = grp.thread_rank();
  const PushTable& T = p.table;
  const unsigned D = T.dim;
  const unsigned long long gid = (blockIdx.x * (unsigned long long)blockDim.x + threadIdx.x) / G;
  const unsigned long long ngroups = (gridDim.x * (unsigned long long)blockDim.x) / G;
  unsigned bits = 0, mx = 0;
  for (unsigned long long u = gid; u < p.rows; u += ngroups) {
    const unsigned long long slot = p.slots[u];
    float* row = T.state + slot * 3ull * D;
    float w[C], m[C], v[C], g[C];
    load_state<G, VEC, ITERS>(gl, row, D, w, m, v);
#pragma unroll
    for (int it = 0; it < ITERS; ++it) {
      const unsigned col = (it * G + gl) * VEC;
#pragma unroll
      for (int x = 0; x < VEC; ++x) {
        const unsigned d = col + x;
        float gv = 0.0f;
        if (d < D) {
          if (p.compact) {
            for (unsigned long long j = p.row_offsets[u]; j < p.row_offsets[u + 1]; ++j)
              gv = __fadd_rn(gv, __fmul_rn(p.source_values[p.source_rows[j] * D + d], p.scales[j]));
            if (!isfinite(gv)) bits |= kRejectReduction;
          } else {
            gv = p.values[u * D + d];
          }
        }
        g[it * VEC + x] = gv;
      }
    }
    bits |= adam_row<G, VEC, ITERS>(gl, T, row, D, g, w, m, v, pass == 1, pass == 0, &mx);
    if (pass == 1 && gl == 0) T.updates[slot] += 1ull;
  }
  bits = cg::reduce(grp, bits, cg::bit_or<unsigned>());
  if (pass == 0 && gl == 0 && bits) atomicOr(p.reject, bits);
  if (pass == 1) {
    mx = cg::reduce(grp, mx, cg::greater<unsigned>());
    if (gl == 0 && mx) atomicMax(&T.dtable->state_absmax_bits, mx);
  }
}

template <int G, int VEC, int ITERS>
cudaError_t run_apply_rows(const ApplyLaunch& p, cudaStream_t s) {
  const unsigned long long groups_per_block = 256 / G;
  const unsigned long long want = (p.rows + groups_per_block - 1) / groups_per_block;
  const unsigned grid = (unsigned)max(1ull, min(want, 148ull * 8));
  apply_rows_kernel<G, VEC, ITERS><<<grid, 256, 0, s>>>(p, 0);
  apply_rows_kernel<G, VEC, ITERS><<<grid, 256, 0, s>>>(p, 1);
  return cudaGetLastError();
}

// ----------------------------------------------------------------- finalize
// Only a push without occurrences launches this kernel; otherwise stage B or C
// finalizes.
__global__ void push_finalize(PushLaunch p) { finalize_tables(p); }

// Persistent grid of the ring kernel: as many blocks as fit on the SMs.
template <int D, typename KeyT>
cudaError_t run_ring(const PushLaunch& p, cudaStream_t s) {
  using S = RingShape<D>;
  static int blocks_per_sm[64] = {};          // per device, set on first use
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  int& bps = blocks_per_sm[dev & 63];
  if (!bps) {
    e = cudaFuncSetAttribute(push_rows_ring<D, KeyT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)S::kBytes);
    if (e != cudaSuccess) return e;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&bps, push_rows_ring<D, KeyT>, S::kWarps * 32,
                                                      S::kBytes);
    if (e != cudaSuccess) return e;
    if (bps < 1) bps = 1;
  }
  int sms = 0;
  e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return e;
  const unsigned long long want = (p.n + 31) / 32;
  const unsigned grid = (unsigned)max(1ull, min(want, (unsigned long long)sms * bps));
  push_rows_ring<D, KeyT><<<grid, S::kWarps * 32, S::kBytes, s>>>(p);
  return cudaGetLastError();
}

template <int G, int VEC, int ITERS, typename KeyT>
cudaError_t run_apply(const PushLaunch& p, cudaStream_t s, int part) {
  if (!p.n) return cudaSuccess;
  constexpr unsigned blocks = (VEC * ITERS <= 4) ? EPS_PUSH_MIN_BLOCKS : 2;
  const unsigned long long want = (p.n + 255) / 256;
  const unsigned grid = (unsigned)max(1ull, min(want, 148ull * blocks));
  const size_t smem = (size_t)(256 / G) * p.dim_max * sizeof(float);
  if (part == 0) {
    if (!p.ring_dim) return cudaSuccess;            // stage A sums the pieces itself
    switch (p.ring_dim) {
      case 32: return run_pieces_uniform<32>(p, s);
      case 64: return run_pieces_uniform<64>(p, s);
      default: return run_pieces_uniform<128>(p, s);
    }
  }
  if (part == 1) {
    if (!p.ring_dim) {
      push_stage_a<G, VEC, ITERS, KeyT><<<grid, 256, 0, s>>>(p);
      return cudaGetLastError();
    }
    switch (p.ring_dim) {
      case 32: return run_ring<32, KeyT>(p, s);
      case 64: return run_ring<64, KeyT>(p, s);
      default: return run_ring<128, KeyT>(p, s);
    }
  }
  push_stage_b<G, VEC, ITERS, KeyT><<<grid, 256, smem, s>>>(p);
  push_stage_c<G, VEC, ITERS, KeyT><<<min(grid, 148u), 256, smem, s>>>(p);
  return cudaGetLastError();
}

template <int G, int VEC, int ITERS>
cudaError_t run_key(const PushLaunch& p, cudaStream_t s, int part) {
  return p.key64 ? run_apply<G, VEC, ITERS, unsigned long long>(p, s, part)
                 : run_apply<G, VEC, ITERS, unsigned int>(p, s, part);
}
}  // namespace

cudaError_t launch_push_prescan(const PushLaunch& p, cudaStream_t stream) {
  // at least 16 values per thread, at most 592 blocks (four per SM): every block
  // ends with atomics on the same words of the control block, which serialise
  // (15,392 blocks took 314 us)
  const unsigned long long want = (p.grad_values + 256ull * 16 - 1) / (256ull * 16);
  const unsigned grid = p.external_reject ? 1u : (unsigned)max(1ull, min(want, 148ull * 4));
  push_prescan<<<grid, 256, 0, stream>>>(p, const_cast<PushTable*>(p.tables));
  return cudaGetLastError();
}

unsigned launch_push_apply_count(const PushLaunch& p, int part) {
  if (!p.n) return 0u;
  if (part == 0) return p.ring_dim ? 1u : 0u;
  return part == 1 ? 1u : 2u;
}
unsigned launch_push_finalize_count(const PushLaunch& p) { return p.n ? 0u : 1u; }

cudaError_t launch_push_apply(const PushLaunch& p, cudaStream_t stream, int part) {
  if (p.vec == 4) {
    switch (p.group) {
      case 8: return run_key<8, 4, 1>(p, stream, part);
      case 16: return run_key<16, 4, 1>(p, stream, part);
      default:
        if (p.iters == 1) return run_key<32, 4, 1>(p, stream, part);
        if (p.iters == 2) return run_key<32, 4, 2>(p, stream, part);
        return run_key<32, 4, 4>(p, stream, part);
    }
  }
  if (p.iters == 1) return run_key<32, 1, 1>(p, stream, part);
  if (p.iters == 2) return run_key<32, 1, 2>(p, stream, part);
  return run_key<32, 1, 4>(p, stream, part);
}

cudaError_t launch_apply_rows(const ApplyLaunch& p, cudaStream_t stream) {
  if (!p.rows) return cudaSuccess;
  if (p.vec == 4) {
    switch (p.group) {
      case 8: return run_apply_rows<8, 4, 1>(p, stream);
      case 16: return run_apply_rows<16, 4, 1>(p, stream);
      default:
        if (p.iters == 1) return run_apply_rows<32, 4, 1>(p, stream);
        if (p.iters == 2) return run_apply_rows<32, 4, 2>(p, stream);
        return run_apply_rows<32, 4, 4>(p, stream);
    }
  }
  if (p.iters == 1) return run_apply_rows<32, 1, 1>(p, stream);
  if (p.iters == 2) return run_apply_rows<32, 1, 2>(p, stream);
  return run_apply_rows<32, 1, 4>(p, stream);
}

cudaError_t launch_push_finalize(const PushLaunch& p, cudaStream_t stream) {
  if (p.n) return cudaSuccess;          // finalized by the apply stages
  push_finalize<<<1, 32, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace eps_b200
