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
//   2. rows pass 0, 3. pieces, 4. long pass 0, 5. rows pass 1, 6. long pass 1,
//   7. finalize  -- advances beta powers and the sequence iff accepted.
//
// Coalescing layout: the occurrences are sorted stably by composite key
// (table rank, slot) and the runs of equal keys are compacted into
// seg_start[U + 1] at lookup time.  `push_rows` gives every coalesced row to a
// group of G lanes (G = D/4: one 128-bit access per lane covers a row): for a
// row with at most 64 occurrences the group issues the row's [w|m|v] loads,
// sums the gradient references serially in occurrence order (bit-exact with the
// reference) with up to 4 gradient rows in flight, and applies LazyAdam in the
// same pass.  A longer (Zipf-head) row reserves ceil(len/64) contiguous piece
// slots; `push_pieces` reduces the pieces in parallel and `push_long` combines
// one row's pieces in piece order on one CTA and applies LazyAdam
// (deterministic; within 1e-6 * sum|terms| of the reference's serial sum).
#include <cooperative_groups.h>
#include <cooperative_groups/reduce.h>

#include "kernels.cuh"

namespace cg = cooperative_groups;

#ifndef EPS_PUSH_DEPTH_REGS
#define EPS_PUSH_DEPTH_REGS 16        // registers per lane for gradient rows in flight
#endif
#ifndef EPS_PUSH_MIN_BLOCKS
#define EPS_PUSH_MIN_BLOCKS 4         // resident 256-thread blocks per SM (C <= 4)
#endif
#ifndef EPS_PIECE_DEPTH_REGS
#define EPS_PIECE_DEPTH_REGS 32       // the same for the long rows' pieces
#endif
#ifndef EPS_PIECE_MIN_BLOCKS
#define EPS_PIECE_MIN_BLOCKS 3
#endif

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
// Grid (x, features): blocks of row y scan feature y's gradient values.
__global__ void __launch_bounds__(256) push_prescan(PushLaunch p, PushTable* tables_rw) {
  __shared__ unsigned s_bad, s_max, s_last;
  if (threadIdx.x == 0) { s_bad = 0; s_max = 0; }
  __syncthreads();
  const PushFeature& F = p.features[blockIdx.y];
  const unsigned long long nvals = F.rows * (unsigned long long)F.dim;
  const unsigned long long stride = (unsigned long long)gridDim.x * blockDim.x;
  unsigned bad = 0;
  float mx = 0.0f;
  if (p.grad_vec4) {
    const float4* g4 = reinterpret_cast<const float4*>(F.grad);
    const unsigned long long n4 = nvals / 4;
#pragma unroll 4
    for (unsigned long long i = blockIdx.x * (unsigned long long)blockDim.x + threadIdx.x; i < n4; i += stride) {
      const float4 x = __ldg(g4 + i);
      bad |= !isfinite(x.x) | !isfinite(x.y) | !isfinite(x.z) | !isfinite(x.w);
      mx = fmaxf(mx, fmaxf(fmaxf(fabsf(x.x), fabsf(x.y)), fmaxf(fabsf(x.z), fabsf(x.w))));
    }
  } else {
    for (unsigned long long i = blockIdx.x * (unsigned long long)blockDim.x + threadIdx.x; i < nvals; i += stride) {
      const float x = __ldg(F.grad + i);
      bad |= !isfinite(x);
      mx = fmaxf(mx, fabsf(x));
    }
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
    s_last = atomicAdd(&p.control->blocks_done, 1u) == gridDim.x * gridDim.y - 1;
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
// owns VEC*ITERS columns), bit-exact with the reference's serial loop.
// The gradient sources of the features are staged in shared memory (row
// pointer and scale index without dependent descriptor loads); up to
// EPS_PUSH_DEPTH_REGS / C gradient rows are in flight; rows past the end add
// -0.0f (the identity).
template <int G, int VEC, int ITERS, int DEPTH_REGS, typename Grp>
__device__ __forceinline__ void reduce_staged(const Grp& grp, const PushLaunch& p,
                                              const float* const* s_grad,
                                              const unsigned long long* s_sbase,
                                              unsigned long long s0, unsigned long long s1,
                                              unsigned D, float (&acc)[VEC * ITERS]) {
  constexpr int C = VEC * ITERS;
  constexpr int DEPTH = G < DEPTH_REGS / C ? G : (DEPTH_REGS / C > 0 ? DEPTH_REGS / C : 1);
  const unsigned gl = grp.thread_rank();
  if (s1 - s0 == 1) {
    // a single term (most rows): 0 + src * scale, every lane reading the source
    const unsigned src = __ldg(p.srcs + s0);
    const unsigned f = src >> kRowBits;
    const unsigned r = src & ((1u << kRowBits) - 1u);
    const float* q = s_grad[f] + (unsigned long long)r * D;
    const float sc = __ldg(p.row_scale + s_sbase[f] + r);
#pragma unroll
    for (int it = 0; it < ITERS; ++it) {
      const unsigned col = (it * G + gl) * VEC;
      float t[VEC];
      if (col < D) load_vec<VEC>(q + col, t);
      else {
#pragma unroll
        for (int v = 0; v < VEC; ++v) t[v] = 0.0f;
      }
#pragma unroll
      for (int v = 0; v < VEC; ++v) acc[it * VEC + v] = __fadd_rn(0.0f, __fmul_rn(t[v], sc));
    }
    return;
  }
#pragma unroll
  for (int k = 0; k < C; ++k) acc[k] = 0.0f;
  for (unsigned long long c0 = s0; c0 < s1; c0 += G) {
    const unsigned long long i = c0 + gl;
    const float* rowp = nullptr;
    float sc = 1.0f;
    if (i < s1) {
      const unsigned src = __ldg(p.srcs + i);
      const unsigned f = src >> kRowBits;
      const unsigned r = src & ((1u << kRowBits) - 1u);
      rowp = s_grad[f] + (unsigned long long)r * D;
      sc = __ldg(p.row_scale + s_sbase[f] + r);
    }
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
      // batch_access.cpp:118: dest += src * scale, in occurrence order
#pragma unroll
      for (int u = 0; u < DEPTH; ++u)
#pragma unroll
        for (int k = 0; k < C; ++k) acc[k] = __fadd_rn(acc[k], __fmul_rn(x[u][k], sv[u]));
    }
  }
}

// Stages every feature's gradient pointer and row-scale base in shared memory.
__device__ __forceinline__ void stage_features(const PushLaunch& p, const float** s_grad,
                                               unsigned long long* s_sbase) {
  for (unsigned f = threadIdx.x; f < p.feature_count; f += blockDim.x) {
    s_grad[f] = p.features[f].grad;
    s_sbase[f] = p.features[f].scale_base;
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
      store_vec<VEC>(row + col, nw);
      store_vec<VEC>(row + D + col, nm);
      store_vec<VEC>(row + 2 * D + col, nv);
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

// --------------------------------------------------------------------- rows
// Coalesced rows come from the lookup's row plan (rows[u], one 16-byte record
// per run of the sorted keys), taken in key order.  A warp takes 32
// consecutive records per step (one load per lane, the next step's records
// loaded one step ahead); its groups of G lanes take the rows round-robin,
// reading the record fields from the owning lane with shuffles.  Every row's
// gradient is one row away: the single occurrence's gradient row times its
// scale (0 + src * scale, batch_access.cpp:118), or, for a row with
// 2..long_run occurrences, its piece sum reduced in occurrence order by
// push_pieces.  The gradient-row, [w|m|v] and counter loads are issued
// together, then LazyAdam.  Padding rows and long rows (push_long) are
// skipped.
template <int G, int VEC, int ITERS, typename KeyT>
__global__ void __launch_bounds__(256, (VEC * ITERS <= 4) ? EPS_PUSH_MIN_BLOCKS : 2) push_rows(PushLaunch p, int pass) {
  __shared__ const float* s_grad[kMaxFeatures];
  const Role R = role(p.control, pass);
  if (!R.run || !(R.apply || R.validate)) return;
  for (unsigned f = threadIdx.x; f < p.feature_count; f += blockDim.x) s_grad[f] = p.features[f].grad;
  __syncthreads();
  constexpr int C = VEC * ITERS;
  constexpr unsigned GPW = 32 / G;            // groups per warp
  const auto grp = cg::tiled_partition<G>(cg::this_thread_block());
  const unsigned gl = grp.thread_rank();
  const unsigned lane = threadIdx.x & 31, gw = lane / G;
  const unsigned U = *(volatile const unsigned*)p.seg_total;
  const unsigned long long warp = (blockIdx.x * (unsigned long long)blockDim.x + threadIdx.x) >> 5;
  const unsigned long long step = ((gridDim.x * (unsigned long long)blockDim.x) >> 5) * 32ull;
  const KeyT smask = slot_mask_of<KeyT>(p.slot_bits);
  unsigned bits = 0;
  int cur_tr = -1;
  unsigned cur_max = 0;
  unsigned long long base = warp * 32ull;
  RowRec nxt{0ull, 0u, kRowSkip};
  if (base + lane < U) nxt = p.rows[base + lane];
  for (; base < U; base += step) {
    const RowRec cur = nxt;
    if (base + step + lane < U) nxt = p.rows[base + step + lane];   // one step ahead
    const unsigned nrow = (unsigned)min(32ull, U - base);
    const unsigned iters = (nrow + GPW - 1) / GPW;
    for (unsigned i = 0; i < iters; ++i) {
      const unsigned j = i * GPW + gw;
      const unsigned jj = j < nrow ? j : 0u;
      const unsigned long long key = __shfl_sync(0xffffffffu, cur.key, jj);
      const unsigned a = __shfl_sync(0xffffffffu, cur.a, jj);
      const unsigned b = __shfl_sync(0xffffffffu, cur.b, jj);
      if (j >= nrow || b == kRowSkip) continue;
      const KeyT K = (KeyT)key;
      const unsigned tr = (unsigned)(K >> p.slot_bits);
      const PushTable& T = p.tables[tr];
      const unsigned D = T.dim;
      const unsigned long long slot = (unsigned long long)(K & smask);
      float* row = T.state + slot * 3ull * D;
      const bool multi = (b & kRowMulti) != 0;
      const float* q = multi ? p.part + (unsigned long long)a * p.dim_max
                             : s_grad[a >> kRowBits] + (unsigned long long)(a & ((1u << kRowBits) - 1u)) * D;
      float t[C], w[C], m[C], v[C], g[C];
#pragma unroll
      for (int it = 0; it < ITERS; ++it) {
        const unsigned col = (it * G + gl) * VEC;
        float x[VEC];
        if (col < D) load_vec<VEC>(q + col, x);
        else {
#pragma unroll
          for (int y = 0; y < VEC; ++y) x[y] = 0.0f;
        }
#pragma unroll
        for (int y = 0; y < VEC; ++y) t[it * VEC + y] = x[y];
      }
      load_state<G, VEC, ITERS>(gl, row, D, w, m, v);
      unsigned long long upd = 0;
      if (R.apply && gl == 0) upd = T.updates[slot];
      if (multi) {
#pragma unroll
        for (int k = 0; k < C; ++k) g[k] = t[k];
      } else {
        const float scale = __uint_as_float(b);
#pragma unroll
        for (int k = 0; k < C; ++k) g[k] = __fadd_rn(0.0f, __fmul_rn(t[k], scale));
      }
      if ((int)tr != cur_tr) {
        if (R.apply) flush_absmax(grp, p, cur_tr, cur_max);
        cur_tr = (int)tr; cur_max = 0;
      }
      bits |= adam_row<G, VEC, ITERS>(gl, T, row, D, g, w, m, v, R.apply, R.validate, &cur_max);
      if (R.apply && gl == 0) T.updates[slot] = upd + 1ull;
    }
  }
  bits = cg::reduce(grp, bits, cg::bit_or<unsigned>());
  if (gl == 0 && bits) atomicOr(&p.control->reject_bits, bits);
  if (R.apply) flush_absmax(grp, p, cur_tr, cur_max);
}

// ------------------------------------------------------------------- pieces
template <int G, int VEC, int ITERS, typename KeyT>
__global__ void __launch_bounds__(256, (VEC * ITERS <= 4) ? EPS_PIECE_MIN_BLOCKS : 2) push_pieces(PushLaunch p, int pass) {
  __shared__ const float* s_grad[kMaxFeatures];
  __shared__ unsigned long long s_sbase[kMaxFeatures];
  const Role R = role(p.control, pass);
  if (!R.run || !R.partials) return;
  constexpr int C = VEC * ITERS;
  stage_features(p, s_grad, s_sbase);
  const auto grp = cg::tiled_partition<G>(cg::this_thread_block());
  const unsigned gl = grp.thread_rank();
  const unsigned count = *(volatile const unsigned*)&p.plan->piece_count;
  const unsigned long long gid = (blockIdx.x * (unsigned long long)blockDim.x + threadIdx.x) / G;
  const unsigned long long ngroups = (gridDim.x * (unsigned long long)blockDim.x) / G;
  for (unsigned long long item = gid; item < count; item += ngroups) {
    const uint2 pc = p.pieces[item];
    const KeyT K = key_at<KeyT>(p.keys, pc.x);
    const unsigned tr = (unsigned)(K >> p.slot_bits);
    if (tr >= p.table_count) continue;
    const unsigned D = p.tables[tr].dim;
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
  const unsigned count = *(volatile const unsigned*)&p.plan->long_count;
  const KeyT smask = slot_mask_of<KeyT>(p.slot_bits);
  unsigned bits = 0;
  unsigned cur_max = 0;
  int cur_tr = -1;
  for (unsigned rec = blockIdx.x; rec < count; rec += gridDim.x) {
    const LongRecord L = p.records[rec];
    const KeyT K = (KeyT)L.key;
    const unsigned tr = (unsigned)(K >> p.slot_bits);
    if (tr >= p.table_count) continue;
    const PushTable& T = p.tables[tr];
    const unsigned D = T.dim;
    const unsigned long long slot = (unsigned long long)(K & smask);
    // a contiguous chunk of pieces per group, combined afterwards in group order
    const unsigned per = (L.npieces + NG - 1) / NG;
    const unsigned p0 = min(L.npieces, per * w), p1 = min(L.npieces, p0 + per);
    float acc[C];
#pragma unroll
    for (int k = 0; k < C; ++k) acc[k] = 0.0f;
    for (unsigned j0 = p0; j0 < p1; j0 += 4) {
      float x[4][C];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const bool use = j0 + u < p1;
        const unsigned long long item = (unsigned long long)L.piece_base + j0 + u;
#pragma unroll
        for (int it = 0; it < ITERS; ++it) {
          const unsigned col = (it * G + gl) * VEC;
          float t[VEC];
          if (use && col < D) load_vec<VEC>(p.part + item * p.dim_max + col, t);
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
  if (!p.n) return cudaSuccess;
  constexpr unsigned rows_blocks = (VEC * ITERS <= 4) ? EPS_PUSH_MIN_BLOCKS : 2;
  constexpr unsigned long long groups_per_block = 256 / G;
  const unsigned long long want = (p.n + groups_per_block - 1) / groups_per_block;
  const unsigned rows_grid = (unsigned)max(1ull, min(want, 148ull * rows_blocks));
  constexpr unsigned piece_blocks = (VEC * ITERS <= 4) ? EPS_PIECE_MIN_BLOCKS : 2;
  const unsigned piece_grid =
      (unsigned)max(1ull, min(((unsigned long long)p.max_pieces + groups_per_block - 1) / groups_per_block,
                              148ull * piece_blocks));
  const size_t long_smem = (size_t)(kLongThreads / G) * p.dim_max * sizeof(float);
  const unsigned long_grid = 148 * 2;
  push_pieces<G, VEC, ITERS, KeyT><<<piece_grid, 256, 0, s>>>(p, 0);
  push_rows<G, VEC, ITERS, KeyT><<<rows_grid, 256, 0, s>>>(p, 0);
  push_long<G, VEC, ITERS, KeyT><<<long_grid, kLongThreads, long_smem, s>>>(p, 0);
  push_rows<G, VEC, ITERS, KeyT><<<rows_grid, 256, 0, s>>>(p, 1);
  push_long<G, VEC, ITERS, KeyT><<<long_grid, kLongThreads, long_smem, s>>>(p, 1);
  return cudaGetLastError();
}

template <int G, int VEC, int ITERS>
cudaError_t run_key(const PushLaunch& p, cudaStream_t s) {
  return p.key64 ? run_apply<G, VEC, ITERS, unsigned long long>(p, s)
                 : run_apply<G, VEC, ITERS, unsigned int>(p, s);
}
}  // namespace

cudaError_t launch_push_prescan(const PushLaunch& p, cudaStream_t stream) {
  // one grid row per feature; enough columns to stream the largest feature
  const unsigned long long per = 256ull * (p.grad_vec4 ? 16 : 4);
  const unsigned long long want = (p.grad_max_values + per - 1) / per;
  const unsigned gx = (unsigned)max(1ull, min(want, 148ull * 4));
  const dim3 grid(gx, max(1u, p.feature_count));
  push_prescan<<<grid, 256, 0, stream>>>(p, const_cast<PushTable*>(p.tables));
  return cudaGetLastError();
}

unsigned launch_push_apply_count(const PushLaunch& p) { return p.n ? 5u : 0u; }

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
  push_finalize<<<1, 32, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace eps_b200
