// Fused compressed all-reduce for DDP gradient buckets (sm_100a).
//
// One kernel per bucket.  Every CTA owns the chunks c = b, b + G, b + 2G, ...
// (8 blocks of 256 elements per chunk, one block per warp), and CTA b of
// every rank owns the same chunks, so the ranks synchronise per CTA
// "column" instead of per chunk:
//
// one-shot
//   phase 1  for each owned chunk: predict (EMA state) -> residual with error
//            feedback -> per-block absmax scale -> Philox stochastic INT4/INT8
//            codes (or per-block top-k selection + index packing) -> chunk
//            record staged in shared memory -> 16-byte P2P stores of the
//            record into every peer's inbox over NVLink
//   signal   one release flag per peer for this column
//   phase 2  one bounded acquire-wait on the peers' column flags, then for
//            each owned chunk: rank-ordered decode + sum of the W records ->
//            predictor add-back -> EMA update -> averaged gradient written
//            back into the bucket
// two-shot (dense modes)
//   phase A  chunk i of the column goes only to its owner rank i mod W
//   phase B  the owner sums its chunks' W records, re-encodes the mean
//            residual as INT8 with per-block scales and pushes that record
//            to every rank
//   phase C  every rank decodes the owners' INT8 records
// single rank (world 1)
//   encode and decode in registers; whole chunks of the gradient, predictor
//   and EF arrive in shared memory by cp.async.bulk on an mbarrier, one
//   chunk ahead (dense modes)
// Chunks chosen as topology passengers are neither encoded nor sent; they
// reconstruct to the prediction and keep their residual as error feedback.
//
// The reference does this work as ~20 eager PyTorch ops, five NCCL
// all_gathers and nine host syncs per bucket
// (python/nangila_ddp/comm_hook.py:125-324).
//
// Every peer access is a plain global load/store through an IPC mapping.
// The only bulk copies (the single-rank prefetch) read this GPU's own
// memory; nothing in this file multicasts.  Every wait is bounded and
// reports through the status word instead of trapping.
#include "fused.h"
#include "ngl_cuda.cuh"

namespace ngl {
namespace dev {

__device__ __forceinline__ int64_t align16(int64_t x) { return (x + 15) & ~int64_t(15); }

__device__ __forceinline__ bool passenger(const Topo& t, int c, int nchunks) {
  return topo_passenger((uint64_t)c, t.a, t.b, t.ndrop, (uint64_t)nchunks);
}


// ------------------------------------------------------------ warp encoders
constexpr int kChunkElems = kChunkBlocks * kBlock;  // 2048

// Where a chunk's inputs are read: global memory (roff = 0) or a shared-
// memory copy of chunk c (pointers to the copy, roff = c * kChunkElems).
template <typename T>
struct ChunkSrc {
  const T* g;
  const float* pred;
  const float* ef;
  int64_t roff;
};

// Residual c = g - pred + e of the lane's 8 consecutive elements of a block.
// kL2Policy compiles the L2-policy loads in (dense modes; the top-k kernels
// keep their registers for the selection).
template <typename T, bool kL2Policy = true>
__device__ __forceinline__ int load_residual(const ChunkSrc<T>& s, int64_t n, int blk, int lane, const QParams& qp,
                                             float (&c)[8]) {
  const int64_t e0 = (int64_t)blk * kBlock + lane * 8;
  const int valid = (int)min64(8, max64(0, n - e0));
  float gv[8], pv[8], ev[8];
  if (kL2Policy && qp.pred_keep > 0.0f && s.roff == 0) {
    // Exchange kernels, global source: the predictor is read again in
    // phase 2, so its lines are kept in L2; gradient and EF stream through.
    const uint64_t stream = l2_policy_evict_first();
    if constexpr (sizeof(T) == 4) load8_policy(reinterpret_cast<const float*>(s.g), e0, valid, stream, gv);
    else load8<T>(s.g, e0, valid, true, gv);
    if (qp.use_pred) load8_policy(s.pred, e0, valid, l2_policy_evict_last(qp.pred_keep), pv);
    if (qp.use_ef) load8_policy(s.ef, e0, valid, stream, ev);
  } else {
    load8<T>(s.g, e0 - s.roff, valid, true, gv);
    if (qp.use_pred) load8<float>(s.pred, e0 - s.roff, valid, true, pv);
    if (qp.use_ef) load8<float>(s.ef, e0 - s.roff, valid, true, ev);
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float p = qp.use_pred ? pv[j] : 0.0f;
    const float e = qp.use_ef ? ev[j] : 0.0f;
    c[j] = (j < valid) ? product_residual(gv[j], p, e) : 0.0f;
  }
  return valid;
}

// Passenger block: the whole residual goes to the error feedback (ef_w).
template <typename T>
__device__ __forceinline__ void passenger_block(const ChunkSrc<T>& s, float* ef_w, int64_t n, int blk, int lane,
                                                const QParams& qp) {
  if (!qp.use_ef) return;
  float cv[8];
  const int valid = load_residual<T, false>(s, n, blk, lane, qp, cv);
  store8<float>(ef_w, (int64_t)blk * kBlock + lane * 8, valid, true, cv);
}

// Double-buffered prefetch of whole chunks (g, pred, ef slices) into dynamic
// shared memory with bulk copies completing on an mbarrier per buffer, so
// the loads of the next owned chunk overlap the current chunk's encode.  A
// partial last chunk is read from global memory instead.  Thread 0 issues;
// every thread waits (bounded) on the buffer's mbarrier phase.
template <typename T>
struct ChunkPipe {
  static constexpr int kG = kChunkElems * (int)sizeof(T);
  static constexpr int kBuf = kG + 2 * kChunkElems * 4;
  static constexpr int kBytes = 2 * kBuf;  // dynamic shared memory
  uint64_t* mbar;                          // 2 mbarriers (static shared)
  uint8_t* buf;
  uint32_t phase = 0;    // bit b: parity of buffer b's next completion
  uint32_t pending = 0;  // bit b: a copy into buffer b is in flight

  __device__ static bool full(int64_t n, int c) { return (int64_t)(c + 1) * kChunkElems <= n; }
  // All threads, once, before the first issue.
  __device__ void init() {
    if (threadIdx.x == 0) {
      mbar_init(&mbar[0], 1);
      mbar_init(&mbar[1], 1);
      fence_mbar_init();
    }
    __syncthreads();
  }
  // All threads (uniform); thread 0 issues the copies of chunk c into buffer b.
  __device__ void issue(const T* g, const float* pred, const float* ef, int c, int b) {
    if (threadIdx.x == 0) {
      uint8_t* d = buf + b * kBuf;
      const int64_t e0 = (int64_t)c * kChunkElems;
      const uint32_t bytes = kG + (pred ? kChunkElems * 4 : 0) + (ef ? kChunkElems * 4 : 0);
      fence_proxy_async_smem();  // earlier generic reads of this buffer before the async writes
      mbar_expect_tx(&mbar[b], bytes);
      bulk_g2s(d, g + e0, kG, &mbar[b]);
      if (pred) bulk_g2s(d + kG, pred + e0, kChunkElems * 4, &mbar[b]);
      if (ef) bulk_g2s(d + kG + kChunkElems * 4, ef + e0, kChunkElems * 4, &mbar[b]);
    }
    pending |= 1u << b;
  }
  // All threads: wait for buffer b; false (uniform) after limit_ns.
  __device__ bool wait(int b, uint64_t limit_ns) {
    const bool ok = mbar_wait(&mbar[b], (phase >> b) & 1u, limit_ns);
    phase ^= 1u << b;
    pending &= ~(1u << b);
    return __syncthreads_or(!ok) == 0;
  }
  // Pointers into buffer b holding chunk c.  Callers pass the result
  // straight to the chunk routine, one call per branch: a source variable
  // merged from this and the global source kept the global base pointer
  // with the buffer's offset (measured on sm_100a), so none is formed.
  __device__ ChunkSrc<T> buffer_source(int b, int c) const {
    const uint8_t* d = buf + b * kBuf;
    return ChunkSrc<T>{reinterpret_cast<const T*>(d), reinterpret_cast<const float*>(d + kG),
                       reinterpret_cast<const float*>(d + kG + kChunkElems * 4), (int64_t)c * kChunkElems};
  }
  // Before leaving early: let copies still in flight land (bounded).
  __device__ void drain(uint64_t limit_ns) {
    for (int b = 0; b < 2; ++b)
      if ((pending >> b) & 1u) mbar_wait(&mbar[b], (phase >> b) & 1u, limit_ns);
    pending = 0;
  }
};

__device__ __forceinline__ float block_absmax(const float (&c)[8]) {
  float m = 0.0f;
#pragma unroll
  for (int j = 0; j < 8; ++j) m = fmaxf(m, fabsf(c[j]));
  return __uint_as_float(__reduce_max_sync(kFull, __float_as_uint(m)));
}

// Dense INT4/INT8 encode of one block: returns the scale; the lane's codes in
// w[0] (INT4) or w[0..1] (INT8); q[] holds the integer codes; writes new EF.
template <int BITS>
__device__ __forceinline__ float encode_dense(const float (&c)[8], int valid, int blk, int lane, const QParams& qp,
                                              float* ef_out, uint32_t (&w)[2], int32_t (&q)[8]) {
  constexpr int32_t qmax = BITS == 4 ? 7 : 127;
  const float s = product_scale(block_absmax(c), (float)qmax);
  const float inv = product_inv(s);
  if (qp.stochastic) {
    const uint32_t g0 = (uint32_t)((int64_t)blk * (kBlock / 4) + lane * 2);
    const U32x4 r0 = product_noise4(qp.seed, qp.rank, qp.bucket, qp.step, g0);
    const U32x4 r1 = product_noise4(qp.seed, qp.rank, qp.bucket, qp.step, g0 + 1);
    const uint32_t rb[8] = {r0.x, r0.y, r0.z, r0.w, r1.x, r1.y, r1.z, r1.w};
#pragma unroll
    for (int j = 0; j < 8; ++j) q[j] = product_code_sr(c[j], inv, u01_from_bits(rb[j]), qmax);
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) q[j] = product_code_rn(c[j], inv, qmax);
  }
  if (qp.use_ef) {
    float e[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) e[j] = NGL_FSUB(c[j], product_deq(q[j], s));
    store8<float>(ef_out, (int64_t)blk * kBlock + lane * 8, valid, true, e);
  }
  if (BITS == 4) {
    uint32_t x = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) x |= ((nib(q[2 * j]) << 4) | nib(q[2 * j + 1])) << (8 * j);
    w[0] = x;
    w[1] = 0;
  } else {
    uint32_t lo = 0, hi = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      lo |= ((uint32_t)q[j] & 0xffu) << (8 * j);
      hi |= ((uint32_t)q[4 + j] & 0xffu) << (8 * j);
    }
    w[0] = lo;
    w[1] = hi;
  }
  return s;
}

// Dense chunk record: [8 x f32 scale][8 x bpb codes]; warp w owns block w.
template <int BITS>
__device__ __forceinline__ void put_dense(uint8_t* rec, int warp, int lane, float s, const uint32_t (&w)[2]) {
  constexpr int bpb = BITS == 4 ? kInt4BlockBytes : kInt8BlockBytes;
  uint8_t* codes = rec + 4 * kChunkBlocks + warp * bpb;
  if (lane == 0) reinterpret_cast<float*>(rec)[warp] = s;
  if (BITS == 4) reinterpret_cast<uint32_t*>(codes)[lane] = w[0];
  else reinterpret_cast<uint2*>(codes)[lane] = make_uint2(w[0], w[1]);
}

// The lane's codes and the scale of warp `warp`'s block in one dense chunk
// record (global memory).
struct DenseLane {
  uint2 x;  // INT4: x.x holds the lane's 8 nibbles; INT8: 8 bytes
  float s;
};
template <int BITS>
__device__ __forceinline__ DenseLane load_dense(const uint8_t* rec, int warp, int lane) {
  constexpr int bpb = BITS == 4 ? kInt4BlockBytes : kInt8BlockBytes;
  const uint8_t* codes = rec + 4 * kChunkBlocks + warp * bpb;
  DenseLane d;
  d.s = __ldcg(reinterpret_cast<const float*>(rec) + warp);
  if (BITS == 4) d.x = make_uint2(__ldcg(reinterpret_cast<const unsigned int*>(codes) + lane), 0u);
  else d.x = __ldcg(reinterpret_cast<const uint2*>(codes) + lane);
  return d;
}
template <int BITS>
__device__ __forceinline__ void accum_lane(const DenseLane& d, float (&acc)[8]) {
  if (BITS == 4) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t byte = (d.x.x >> (8 * j)) & 0xffu;
      acc[2 * j] = product_accum(acc[2 * j], sext4(byte >> 4), d.s);
      acc[2 * j + 1] = product_accum(acc[2 * j + 1], sext4(byte & 0xfu), d.s);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      acc[j] = product_accum(acc[j], (int32_t)(int8_t)((d.x.x >> (8 * j)) & 0xffu), d.s);
      acc[4 + j] = product_accum(acc[4 + j], (int32_t)(int8_t)((d.x.y >> (8 * j)) & 0xffu), d.s);
    }
  }
}
// Accumulate warp `warp`'s block of one dense chunk record (global memory).
template <int BITS>
__device__ __forceinline__ void accum_dense(const uint8_t* rec, int warp, int lane, float (&acc)[8]) {
  accum_lane<BITS>(load_dense<BITS>(rec, warp, lane), acc);
}
// The same over `world` records (rec_of(src), src = 0 .. world-1), four
// ranks at a time: a group's loads are all issued before its first sum, so
// their round trips overlap (two instead of eight at eight ranks, with 8-12
// more live registers rather than 16-24); the sums run in rank order (the
// same FMA sequence as one record at a time).
constexpr int kRankGroup = 4;
template <int BITS, typename RecOf>
__device__ __forceinline__ void accum_dense_ranks(const RecOf& rec_of, int world, int warp, int lane,
                                                  float (&acc)[8]) {
  for (int g0 = 0; g0 < world; g0 += kRankGroup) {
    DenseLane d[kRankGroup];
#pragma unroll
    for (int i = 0; i < kRankGroup; ++i)
      if (g0 + i < world) d[i] = load_dense<BITS>(rec_of(g0 + i), warp, lane);
#pragma unroll
    for (int i = 0; i < kRankGroup; ++i)
      if (g0 + i < world) accum_lane<BITS>(d[i], acc);
  }
}

// ------------------------------------------------------ fused optimizer
// One AdamW step of parameter element x with gradient g (decoupled weight
// decay, bias-corrected moments; see OptParams).
__device__ __forceinline__ void adamw1(const OptParams& o, float g, float& x, float& m, float& v) {
  x = x * o.decay;
  m = o.beta1 * m + (1.0f - o.beta1) * g;
  v = o.beta2 * v + (1.0f - o.beta2) * (g * g);
  const float denom = sqrtf(v) * o.inv_bc2_sqrt + o.eps;
  x = x - o.step_size * (m / denom);
}

// Index of the segment holding bucket element e (the last with off <= e).
__device__ __forceinline__ int opt_seg(const OptParams& o, int64_t e) {
  int lo = 0, hi = o.nsegs - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (__ldg(&o.segs[mid].off) <= e) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

// AdamW on the lane's 8 averaged gradients (elements e0 .. e0 + valid - 1 of
// this launch).  Whole vectors when the 8 lie in one parameter at a 16-byte
// boundary (every GPT-2 / Llama parameter has a multiple of 8 elements);
// element by element otherwise.  Elements outside every segment are skipped.
__device__ __forceinline__ void adamw8(const OptParams& o, int64_t e0, int valid, const float (&g)[8]) {
  const int64_t b0 = o.base + e0;
  const int si = opt_seg(o, b0);
  const OptSeg s = o.segs[si];
  const int64_t rel = b0 - s.off;
  if (valid == 8 && rel >= 0 && rel + 8 <= s.numel && (rel & 7) == 0 &&
      ((reinterpret_cast<uintptr_t>(s.p) | reinterpret_cast<uintptr_t>(s.m) | reinterpret_cast<uintptr_t>(s.v)) &
       15u) == 0) {
    float x[8], m[8], v[8];
    load8<float>(s.p, rel, 8, true, x);
    load8<float>(s.m, rel, 8, true, m);
    load8<float>(s.v, rel, 8, true, v);
#pragma unroll
    for (int j = 0; j < 8; ++j) adamw1(o, g[j], x[j], m[j], v[j]);
    store8<float>(s.p, rel, 8, true, x);
    store8<float>(s.m, rel, 8, true, m);
    store8<float>(s.v, rel, 8, true, v);
    return;
  }
  for (int j = 0; j < valid; ++j) {
    const int sj = opt_seg(o, b0 + j);
    const OptSeg t = o.segs[sj];
    const int64_t r = b0 + j - t.off;
    if (r < 0 || r >= t.numel) continue;
    float x = t.p[r], m = t.m[r], v = t.v[r];
    adamw1(o, g[j], x, m, v);
    t.p[r] = x;
    t.m[r] = m;
    t.v[r] = v;
  }
}

// avg = pred + acc / W -> bucket; EMA update of the predictor state; with
// kOpt, AdamW on the bucket's parameters from the averaged gradient.
template <typename T, bool kL2Policy = true, bool kOpt = false>
__device__ __forceinline__ void finalize(T* grad, float* pred, int64_t n, int blk, int lane, const float (&acc)[8],
                                         const FParams& fp) {
  const int64_t e0 = (int64_t)blk * kBlock + lane * 8;
  const int valid = (int)min64(8, max64(0, n - e0));
  if (valid <= 0) return;
  float p[8], avg[8];
  if (fp.use_pred) {
    if (kL2Policy && fp.pred_stream) load8_policy(pred, e0, valid, l2_policy_evict_first(), p);
    else load8<float>(pred, e0, valid, true, p);
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    if (!fp.use_pred) p[j] = 0.0f;
    avg[j] = product_average(p[j], acc[j], fp.inv_world);
  }
  store8<T>(grad, e0, valid, true, avg);
  if constexpr (kOpt) adamw8(fp.opt, e0, valid, avg);
  if (fp.use_pred) {
#pragma unroll
    for (int j = 0; j < 8; ++j) p[j] = product_ema(p[j], avg[j], fp.beta, fp.omb, fp.first != 0);
    store8<float>(pred, e0, valid, true, p);
  }
}

// --------------------------------------------------------------- top-k warp
// Warp sums of |{m >= c1}|, |{m >= c2}|, |{m >= c3}| over the block, as
// three 10-bit fields of one word (each count is at most 256).
__device__ __forceinline__ uint32_t count_ge3(const uint32_t (&m)[8], uint32_t c1, uint32_t c2, uint32_t c3) {
  uint32_t l = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j)
    l += (uint32_t)(m[j] >= c1) | ((uint32_t)(m[j] >= c2) << 10) | ((uint32_t)(m[j] >= c3) << 20);
  return __reduce_add_sync(kFull, l);
}

// Selection threshold of one 256-block from the |c| bit patterns m (bit 31
// clear, so the unsigned order is the order of |c|; NaN sorts above inf):
// either the keff-th largest pattern, or a T with exactly keff patterns
// >= T.  Both keep the same set as the host's bitwise search for the
// largest T with |{m >= T}| >= keff, after the tie handling of the caller.
//
// Bracket search: lo always has |{m >= lo}| >= keff and hi has fewer.  The
// first round tests three patterns half a binade, one and two binades
// below the block maximum M together (three counts in one warp sum): the
// kept fraction of a gradient block mostly lies there, so one round
// narrows [0, M] to a quarter binade.  Later rounds split [lo, hi) in four
// the same way, until hi = lo + 1 or exactly keff patterns are >= lo.
// This takes about 4-6 dependent warp sums on gradient blocks instead of
// the ~14 of a bit-at-a-time search.
__device__ __forceinline__ uint32_t topk_threshold_bits(const uint32_t (&m)[8], int keff, uint32_t& M) {
  uint32_t mx = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) mx = max(mx, m[j]);
  M = __reduce_max_sync(kFull, mx);
  if (keff <= 0) return 0xffffffffu;  // nothing is >= it: no element kept
  uint32_t lo = 0, hi = M + 1;  // M <= 0x7fffffff
  bool first = true;
  while (hi - lo > 1) {
    uint32_t c1, c2, c3;
    if (first) {
      c3 = M > (1u << 22) ? M - (1u << 22) : 0u;
      c2 = M > (1u << 23) ? M - (1u << 23) : 0u;
      c1 = M > (2u << 23) ? M - (2u << 23) : 0u;
      first = false;
    } else {
      const uint32_t d = hi - lo;
      c1 = lo + (d >> 2);
      c2 = lo + (d >> 1);  // lo < c2 < hi: every round makes progress
      c3 = hi - (d >> 2);
    }
    const uint32_t s = count_ge3(m, c1, c2, c3);
    const int n1 = (int)(s & 1023u), n2 = (int)((s >> 10) & 1023u), n3 = (int)(s >> 20);
    int nlo = -1;
    if (n3 >= keff) {
      lo = c3;
      nlo = n3;
    } else if (n2 >= keff) {
      lo = c2;
      hi = c3;
      nlo = n2;
    } else if (n1 >= keff) {
      lo = c1;
      hi = c2;
      nlo = n1;
    } else {
      hi = c1;
    }
    if (nlo == keff) break;
  }
  return lo;
}

struct TopkSel {
  float s;
  uint32_t selmask;  // bit j: element j of this lane kept
  int32_t q[8];
};

// Keep the k largest |c| of one block (ties -> lower index), int8 codes with
// scale absmax/127, record [f32 s][k idx ascending][k int8] written to `rec`
// (shared memory of this warp), new EF written.
__device__ __forceinline__ TopkSel topk_select(const float (&c)[8], int valid, int blk, int lane, int k, int64_t n,
                                               const QParams& qp, float* ef_out, uint8_t* rec, int rec_bytes) {
  TopkSel r;
  const int len = (int)min64(kBlock, n - (int64_t)blk * kBlock);
  const int keff = min(k, len);
  uint32_t m[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) m[j] = __float_as_uint(fabsf(c[j]));
  uint32_t M;  // largest |c| bit pattern of the block (NaN above inf)
  const uint32_t T = topk_threshold_bits(m, keff, M);
  int gt = 0, eq = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    gt += (m[j] > T);
    eq += (m[j] == T && j < valid);
  }
  const int budget = keff - (int)__reduce_add_sync(kFull, (unsigned)gt);
  int eq_rank = warp_excl_scan(eq, lane);
  uint32_t sel = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    bool sj = m[j] > T;
    if (!sj && m[j] == T && j < valid) {
      sj = eq_rank < budget;
      ++eq_rank;
    }
    sel |= (uint32_t)sj << j;
  }
  const int out_base = warp_excl_scan(__popc(sel), lane);
  // the block's absmax is the largest pattern when no |c| is NaN (maxNum
  // folds skip NaN, so a NaN block takes the full fold)
  r.s = product_scale(M <= 0x7f800000u ? __uint_as_float(M) : block_absmax(c), 127.0f);
  const float inv = product_inv(r.s);
  for (int w = lane; w < rec_bytes / 4; w += 32) reinterpret_cast<uint32_t*>(rec)[w] = 0u;
  __syncwarp();
  if (lane == 0) reinterpret_cast<float*>(rec)[0] = r.s;
  int pos = out_base;
  float e[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    r.q[j] = 0;
    e[j] = c[j];
    if ((sel >> j) & 1u) {
      r.q[j] = product_code_rn(c[j], inv, 127);
      rec[4 + pos] = (uint8_t)(lane * 8 + j);
      rec[4 + k + pos] = (uint8_t)(int8_t)r.q[j];
      e[j] = NGL_FSUB(c[j], product_deq(r.q[j], r.s));
      ++pos;
    }
  }
  r.selmask = sel;
  if (qp.use_ef) store8<float>(ef_out, (int64_t)blk * kBlock + lane * 8, valid, true, e);
  __syncwarp();
  return r;
}

// Add one rank's block record (global memory) into the warp accumulator,
// staging it through shared memory.
__device__ __forceinline__ void topk_accum_global(const uint8_t* rec_g, uint8_t* stage, int k, int keff,
                                                  int rec_bytes, float* acc, int lane) {
  for (int w = lane; w < rec_bytes / 4; w += 32)
    reinterpret_cast<uint32_t*>(stage)[w] = __ldcg(reinterpret_cast<const unsigned int*>(rec_g) + w);
  __syncwarp();
  const float s = reinterpret_cast<const float*>(stage)[0];
  for (int j = lane; j < keff; j += 32) {
    const int idx = stage[4 + j];
    acc[idx] = product_accum(acc[idx], (int32_t)(int8_t)stage[4 + k + j], s);
  }
  __syncwarp();
}

// Add `world` ranks' records of one block (rec_of(src) + block offset, global
// memory) into the warp accumulator `acc` (shared memory), in rank order.
// A record of R = rec_bytes / 4 <= 32 words is read with one load per lane
// and rank, all issued before the first sum; each kept entry's index and
// code bytes then reach their lane by shuffles.  Longer records (k > 62)
// are staged rank by rank.
template <typename RecOf>
__device__ __forceinline__ void topk_accum_ranks(const RecOf& rec_of, int world, int64_t boff, uint8_t* stage, int k,
                                                 int keff, int rec_bytes, float* acc, int lane) {
  const int R = rec_bytes >> 2;
  if (R > 32) {
    for (int src = 0; src < world; ++src) topk_accum_global(rec_of(src) + boff, stage, k, keff, rec_bytes, acc, lane);
    return;
  }
  uint32_t wv[kMaxWorld];
#pragma unroll
  for (int src = 0; src < kMaxWorld; ++src)
    wv[src] = (src < world && lane < R) ? __ldcg(reinterpret_cast<const unsigned int*>(rec_of(src) + boff) + lane)
                                        : 0u;
#pragma unroll
  for (int src = 0; src < kMaxWorld; ++src) {
    if (src >= world) break;
    const float s = __uint_as_float(__shfl_sync(kFull, wv[src], 0));
    for (int base = 0; base < keff; base += 32) {
      const int j = base + lane;
      const int bi = 4 + j, bq = 4 + k + j;  // byte offsets of entry j's index and code
      const uint32_t wi = __shfl_sync(kFull, wv[src], min(bi >> 2, 31));
      const uint32_t wq = __shfl_sync(kFull, wv[src], min(bq >> 2, 31));
      if (j < keff) {
        const int idx = (int)((wi >> (8 * (bi & 3))) & 0xffu);
        const int32_t q = (int32_t)(int8_t)((wq >> (8 * (bq & 3))) & 0xffu);
        acc[idx] = product_accum(acc[idx], q, s);
      }
    }
    __syncwarp();  // this rank's sums land before the next rank's
  }
}

// ------------------------------------------------------------- chunk level
// Encode chunk c into the shared-memory record `rec` (all threads; ends
// with __syncthreads).  Blocks past the end are written as empty blocks.
template <int MODE, typename T>
__device__ __forceinline__ void encode_chunk(const ChunkSrc<T>& src, float* ef_w, int64_t n, int nblk, int nchunks,
                                             int k, int rec_bytes, const QParams& qp, int c, uint8_t* rec) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int blk = c * kChunkBlocks + warp;
  if (passenger(qp.topo, c, nchunks)) {
    // No record is sent for a passenger; the zero record (which decodes to
    // zero) is staged for the single-GPU encode path.
    if (blk < nblk) passenger_block<T>(src, ef_w, n, blk, lane, qp);
    const int bytes = chunk_record_bytes(MODE, k);
    for (int w = threadIdx.x; w < bytes / 4; w += blockDim.x) reinterpret_cast<uint32_t*>(rec)[w] = 0u;
    __syncthreads();
    return;
  }
  if (MODE == kTopK) {
    uint8_t* r = rec + warp * rec_bytes;
    if (blk < nblk) {
      float cv[8];
      const int valid = load_residual<T, false>(src, n, blk, lane, qp, cv);
      topk_select(cv, valid, blk, lane, k, n, qp, ef_w, r, rec_bytes);
    } else {
      for (int w = lane; w < rec_bytes / 4; w += 32) reinterpret_cast<uint32_t*>(r)[w] = 0u;
    }
  } else {
    constexpr int BITS = MODE == kInt4 ? 4 : 8;
    uint32_t w[2] = {0u, 0u};
    float s = 0.0f;
    if (blk < nblk) {
      float cv[8];
      int32_t q[8];
      const int valid = load_residual<T>(src, n, blk, lane, qp, cv);
      s = encode_dense<BITS>(cv, valid, blk, lane, qp, ef_w, w, q);
    }
    put_dense<BITS>(rec, warp, lane, s, w);
  }
  __syncthreads();
}

// Phase 1 of the exchange kernels, one warp: encode block `warp` of chunk c
// and store this block's part of the chunk record straight into each of
// `ndst` destination chunk records (dst(i), i = 0 .. ndst-1): no CTA-wide
// staging, so warps go through their chunks independently.  Dense blocks:
// the scale (lane 0) and the lane's code word, coalesced across the warp.
// Top-k blocks: the record is assembled in the warp's shared-memory slot
// `wrec`, then copied out in 16-byte (or 4-byte) words.  Blocks past the
// end are written as empty blocks; a passenger chunk writes nothing (its
// residual goes to the error feedback).  The layout is encode_chunk's.
// Inputs are read with direct loads: the prefetch pipeline of the
// single-rank kernel measured slower here, since the exchange phases want
// the occupancy its buffers would take.
template <int MODE, typename T, typename Dst>
__device__ __forceinline__ void encode_push_block(const FusedParams& P, int c, uint8_t* wrec, int ndst,
                                                  const Dst& dst) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int blk = c * kChunkBlocks + warp;
  const ChunkSrc<T> src{reinterpret_cast<const T*>(P.grad), P.pred, P.ef, 0};
  if (passenger(P.q.topo, c, P.nchunks)) {
    if (blk < P.nblk) passenger_block<T>(src, P.ef, P.n, blk, lane, P.q);
    return;
  }
  if constexpr (MODE == kTopK) {
    if (blk < P.nblk) {
      float cv[8];
      const int valid = load_residual<T, false>(src, P.n, blk, lane, P.q, cv);
      topk_select(cv, valid, blk, lane, P.k, P.n, P.q, P.ef, wrec, P.rec_bytes);
    } else {
      for (int w = lane; w < P.rec_bytes / 4; w += 32) reinterpret_cast<uint32_t*>(wrec)[w] = 0u;
      __syncwarp();
    }
    const int64_t boff = (int64_t)warp * P.rec_bytes;
    if ((P.rec_bytes & 15) == 0) {
      const int Q = P.rec_bytes >> 4;
      for (int i = lane; i < Q * ndst; i += 32) {
        const int d = i / Q, q = i - d * Q;
        reinterpret_cast<uint4*>(dst(d) + boff)[q] = reinterpret_cast<const uint4*>(wrec)[q];
      }
    } else {
      const int Q = P.rec_bytes >> 2;
      for (int i = lane; i < Q * ndst; i += 32) {
        const int d = i / Q, q = i - d * Q;
        reinterpret_cast<uint32_t*>(dst(d) + boff)[q] = reinterpret_cast<const uint32_t*>(wrec)[q];
      }
    }
    __syncwarp();  // the slot is read out before the next block rewrites it
  } else {
    constexpr int BITS = MODE == kInt4 ? 4 : 8;
    constexpr int bpb = BITS == 4 ? kInt4BlockBytes : kInt8BlockBytes;
    uint32_t w[2] = {0u, 0u};
    float s = 0.0f;
    if (blk < P.nblk) {
      float cv[8];
      int32_t q[8];
      const int valid = load_residual<T>(src, P.n, blk, lane, P.q, cv);
      s = encode_dense<BITS>(cv, valid, blk, lane, P.q, P.ef, w, q);
    }
    for (int d = 0; d < ndst; ++d) {
      uint8_t* rec = dst(d);
      uint8_t* codes = rec + 4 * kChunkBlocks + warp * bpb;
      if (lane == 0) reinterpret_cast<float*>(rec)[warp] = s;
      if (BITS == 4) reinterpret_cast<uint32_t*>(codes)[lane] = w[0];
      else reinterpret_cast<uint2*>(codes)[lane] = make_uint2(w[0], w[1]);
    }
  }
}

__device__ __forceinline__ void copy_record(uint8_t* dst, const uint8_t* rec, int bytes) {
  const uint4* s = reinterpret_cast<const uint4*>(rec);
  uint4* d = reinterpret_cast<uint4*>(dst);
  for (int i = threadIdx.x; i < bytes / 16; i += blockDim.x) d[i] = s[i];
}

// Decode chunk c: accumulate the W records in rank order, finalize.
template <int MODE, typename T, bool kOpt, typename RecOf>
__device__ __forceinline__ void decode_chunk(const RecOf& rec_of, int world, T* grad, float* pred, int64_t n, int nblk,
                                             int nchunks, int k, int rec_bytes, const FParams& fp, int c,
                                             uint8_t* stage_smem, float* acc_smem) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int blk = c * kChunkBlocks + warp;
  if (blk >= nblk) return;
  float acc[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j] = 0.0f;
  if (passenger(fp.topo, c, nchunks)) {
    // nothing was sent: the passenger reconstructs to the prediction
  } else if (MODE == kTopK) {
    float* a = acc_smem + warp * kBlock;
    uint8_t* stage = stage_smem + warp * kTopkMaxRec;
#pragma unroll
    for (int j = 0; j < 8; ++j) a[lane * 8 + j] = 0.0f;
    __syncwarp();
    const int keff = min(k, (int)min64(kBlock, n - (int64_t)blk * kBlock));
    topk_accum_ranks(rec_of, world, (int64_t)warp * rec_bytes, stage, k, keff, rec_bytes, a, lane);
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = a[lane * 8 + j];
    __syncwarp();
  } else {
    constexpr int BITS = MODE == kInt4 ? 4 : 8;
    accum_dense_ranks<BITS>(rec_of, world, warp, lane, acc);
  }
  finalize<T, MODE != kTopK, kOpt>(grad, pred, n, blk, lane, acc, fp);
}

// ---------------------------------------------------------- flag addressing
__device__ __forceinline__ uint64_t* col_flag(const FusedParams& P, int r, int kind, int src, int col) {
  return reinterpret_cast<uint64_t*>(P.sym[r] + P.flags_off) +
         ((int64_t)((P.parity * 2 + kind) * P.world + src) * kMaxCols + col);
}
__device__ __forceinline__ uint8_t* slot_rec(const FusedParams& P, int r, int src, int c) {
  return P.sym[r] + P.inbox_off + (int64_t)(P.parity * P.world + src) * P.slot_bytes + (int64_t)c * P.chunk_bytes;
}
__device__ __forceinline__ uint8_t* result_rec(const FusedParams& P, int r, int c) {
  return P.sym[r] + P.result_off + (int64_t)P.parity * P.result_bytes +
         (int64_t)c * chunk_record_bytes(kInt8, 0);
}
__device__ __forceinline__ void st_release_u64(uint64_t* p, uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_acquire_u64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
// The flag carries the epoch (low word) and a tag of (bucket size, bucket
// id, grid) so ranks that disagree are reported instead of mixing buckets.
__device__ __forceinline__ uint32_t flag_tag(const FusedParams& P) { return P.tag ^ (gridDim.x * 0x9E3779B1u); }
__device__ __forceinline__ uint64_t flag_value(const FusedParams& P) {
  return ((uint64_t)flag_tag(P) << 32) | P.epoch;
}

// Wait for a flag of this epoch and check its tag: 0 ok, -1 timeout,
// -2 another CTA failed, 1 tag mismatch.
__device__ int wait_tagged(const FusedParams& P, const uint64_t* f) {
  uint64_t v = ld_acquire_u64(f);
  if ((uint32_t)v != P.epoch) {
    const uint64_t t0 = globaltimer();
    uint32_t spins = 0;
    while (true) {
      __nanosleep(32);
      v = ld_acquire_u64(f);
      if ((uint32_t)v == P.epoch) break;
      if ((++spins & 31u) == 0) {
        if (globaltimer() - t0 > P.timeout_ns) return -1;
        if (ld_volatile_i32(P.status) != 0) return -2;
      }
    }
  }
  return ((uint32_t)(v >> 32) == flag_tag(P)) ? 0 : 1;
}

// Release this CTA's column flag of `kind` on every peer (after a barrier
// that orders all of the CTA's stores before it).
__device__ __forceinline__ void signal_column(const FusedParams& P, int kind) {
  __syncthreads();
  const int t = threadIdx.x;
  if (t < P.world && t != P.rank) {
    __threadfence_system();
    st_release_u64(col_flag(P, t, kind, P.rank, blockIdx.x), flag_value(P));
  }
}

// All threads: wait for every peer's column flag of `kind`.  Returns false
// (uniformly) if the CTA must stop.
__device__ bool wait_column(const FusedParams& P, int kind, int* s_abort) {
  const int t = threadIdx.x;
  if (t < P.world && t != P.rank) {
    const int rc = wait_tagged(P, col_flag(P, P.rank, kind, t, blockIdx.x));
    if (rc != 0) {
      if (rc == -1) set_status(P.status, kind == kFlagPayload ? kTimeoutPayload : kTimeoutResult, blockIdx.x, t);
      else if (rc == 1) set_status(P.status, kBadHeader, blockIdx.x, t);
      atomicExch(s_abort, 1);
    }
  }
  __syncthreads();
  return *s_abort == 0;
}

// ------------------------------------------------------------------ kernels
// Per-warp top-k record slot in shared memory: the largest record rounded up
// to 16 bytes, so every slot starts on a 16-byte boundary (the one-shot
// kernel copies records out of it in 16-byte words).
constexpr int kTopkSlot = (kTopkMaxRec + 15) / 16 * 16;
static_assert(kWarps * kTopkSlot >= kMaxChunkRec, "the slots also hold one whole chunk record");

template <int MODE>
struct Smem {
  // encode_chunk's chunk record (the encode kernel); the one-shot kernel
  // uses it as per-warp top-k record slots (kTopkSlot bytes each)
  static constexpr int kRec = MODE == kTopK ? kWarps * kTopkSlot : (MODE == kInt4 ? 1056 : 2080);
  static constexpr int kStage = MODE == kTopK ? kWarps * kTopkMaxRec : 16;
  static constexpr int kAcc = MODE == kTopK ? kWarps * kBlock : 4;
};

// Top-k: 64 registers without spills (four CTAs per SM instead of three at
// 80); the dense instances keep the compiler's choice.
template <int MODE, typename T, bool kOpt>
__global__ void __launch_bounds__(kThreads, MODE == kTopK ? 4 : 0) oneshot_kernel(FusedParams P) {
  __shared__ int s_abort;
  __shared__ __align__(16) uint8_t rec[Smem<MODE>::kRec];
  __shared__ __align__(16) uint8_t stage[Smem<MODE>::kStage];
  __shared__ __align__(16) float acc_smem[Smem<MODE>::kAcc];
  if (threadIdx.x == 0) s_abort = 0;
  // Debug builds: every record of this launch fits its inbox slot, and every
  // rank's region is mapped.
  NGL_BOUNDS_UNIFORM((int64_t)P.nchunks * P.chunk_bytes <= P.slot_bytes && P.world <= kMaxWorld, P.status,
                     P.nchunks, P.chunk_bytes);
  for (int r = 0; r < P.world; ++r) NGL_BOUNDS_UNIFORM(P.sym[r] != nullptr, P.status, -2, r);
  // Phase 1: each warp encodes its block of every owned chunk and pushes
  // it to every rank (self last).
  uint8_t* wrec = rec + (threadIdx.x >> 5) * kTopkSlot;
  for (int c = blockIdx.x; c < P.nchunks; c += gridDim.x)
    encode_push_block<MODE, T>(P, c, wrec, P.world,
                               [&](int i) { return slot_rec(P, (P.rank + 1 + i) % P.world, P.rank, c); });
  signal_column(P, kFlagPayload);
  // Phase 2: wait for the peers' records of this column, reduce.
  if (!wait_column(P, kFlagPayload, &s_abort)) return;
  auto rec_of = [&](int src) { return slot_rec(P, P.rank, src, 0); };
  for (int c = blockIdx.x; c < P.nchunks; c += gridDim.x) {
    auto rc = [&](int src) { return rec_of(src) + (int64_t)c * P.chunk_bytes; };
    decode_chunk<MODE, T, kOpt>(rc, P.world, reinterpret_cast<T*>(P.grad), P.pred, P.n, P.nblk, P.nchunks, P.k,
                          P.rec_bytes, P.f, c, stage, acc_smem);
  }
}

template <int MODE, typename T, bool kOpt>
__global__ void __launch_bounds__(kThreads) twoshot_kernel(FusedParams P) {
  constexpr int BITS = MODE == kInt4 ? 4 : 8;
  __shared__ int s_abort;
  if (threadIdx.x == 0) s_abort = 0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  NGL_BOUNDS_UNIFORM((int64_t)P.nchunks * P.chunk_bytes <= P.slot_bytes &&
                         (int64_t)P.nchunks * chunk_record_bytes(kInt8, 0) <= P.result_bytes && P.world <= kMaxWorld,
                     P.status, P.nchunks, P.chunk_bytes);
  for (int r = 0; r < P.world; ++r) NGL_BOUNDS_UNIFORM(P.sym[r] != nullptr, P.status, -2, r);
  // Phase A: chunk i of this column goes to its owner rank i mod W (each
  // warp pushes its own block).
  {
    int i = 0;
    for (int c = blockIdx.x; c < P.nchunks; c += gridDim.x, ++i)
      encode_push_block<MODE, T>(P, c, nullptr, 1, [&](int) { return slot_rec(P, i % P.world, P.rank, c); });
  }
  signal_column(P, kFlagPayload);
  if (!wait_column(P, kFlagPayload, &s_abort)) return;
  // Phase B: reduce owned chunks, re-encode the mean residual as INT8.
  {
    int i = 0;
    for (int c = blockIdx.x; c < P.nchunks; c += gridDim.x, ++i) {
      if (i % P.world != P.rank || passenger(P.q.topo, c, P.nchunks)) continue;
      const int blk = c * kChunkBlocks + warp;
      float acc[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = 0.0f;
      if (blk < P.nblk)
        accum_dense_ranks<BITS>([&](int src) { return slot_rec(P, P.rank, src, c); }, P.world, warp, lane, acc);
      float m[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) m[j] = NGL_FMUL(acc[j], P.f.inv_world);
      const float s2 = product_scale(block_absmax(m), 127.0f);
      const float inv2 = product_inv(s2);
      uint32_t w[2] = {0u, 0u};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        w[0] |= ((uint32_t)product_code_rn(m[j], inv2, 127) & 0xffu) << (8 * j);
        w[1] |= ((uint32_t)product_code_rn(m[4 + j], inv2, 127) & 0xffu) << (8 * j);
      }
      // this warp's block of the INT8 result record, to every rank (self last)
      for (int t = 0; t < P.world; ++t) put_dense<8>(result_rec(P, (P.rank + 1 + t) % P.world, c), warp, lane, s2, w);
    }
  }
  signal_column(P, kFlagResult);
  if (!wait_column(P, kFlagResult, &s_abort)) return;
  // Phase C: decode the owners' INT8 records.
  FParams f = P.f;
  f.inv_world = 1.0f;
  for (int c = blockIdx.x; c < P.nchunks; c += gridDim.x) {
    const int blk = c * kChunkBlocks + warp;
    if (blk >= P.nblk) continue;
    float acc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = 0.0f;
    if (!passenger(P.f.topo, c, P.nchunks)) accum_dense<8>(result_rec(P, P.rank, c), warp, lane, acc);
    finalize<T, true, kOpt>(reinterpret_cast<T*>(P.grad), P.pred, P.n, blk, lane, acc, f);
  }
}

// One chunk of the single-rank kernel: encode + decode in registers.
template <int MODE, typename T, bool kOpt>
__device__ __forceinline__ void single_chunk(const FusedParams& P, const ChunkSrc<T>& in, int ch, uint8_t* rec_smem) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int blk = ch * kChunkBlocks + warp;
  if (blk >= P.nblk) return;
  float c[8], acc[8];
  const int valid = load_residual<T, false>(in, P.n, blk, lane, P.q, c);
  if (passenger(P.q.topo, ch, P.nchunks)) {
    if (P.q.use_ef) store8<float>(P.ef, (int64_t)blk * kBlock + lane * 8, valid, true, c);
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = 0.0f;
  } else if (MODE == kTopK) {
    TopkSel r = topk_select(c, valid, blk, lane, P.k, P.n, P.q, P.ef, rec_smem + warp * kTopkMaxRec, P.rec_bytes);
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = ((r.selmask >> j) & 1u) ? product_accum(0.0f, r.q[j], r.s) : 0.0f;
  } else {
    constexpr int BITS = MODE == kInt4 ? 4 : 8;
    uint32_t w[2];
    int32_t q[8];
    const float s = encode_dense<BITS>(c, valid, blk, lane, P.q, P.ef, w, q);
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = product_accum(0.0f, q[j], s);
  }
  finalize<T, false, kOpt>(reinterpret_cast<T*>(P.grad), P.pred, P.n, blk, lane, acc, P.f);
}

// Single rank: encode + decode in registers (no exchange); inputs of whole
// chunks through the prefetch pipeline.
// Which kernels read their inputs through the prefetch pipeline (measured
// per kernel on B200, 64M-element buckets): the dense single-rank kernel
// gains; the exchange kernels and top-k, which need their occupancy, lose.
template <int MODE, bool kExchange>
inline constexpr bool kPrefetch = !kExchange && MODE != kTopK;

// Top-k: 64 registers without spills, four CTAs per SM (0.42 ms at 64M
// elements against 0.46 ms at 76 registers and three).  The one-shot top-k
// kernel spills at 64 and is no faster, so it keeps the default bound.
template <int MODE, typename T, bool kOpt>
__global__ void __launch_bounds__(kThreads, MODE == kTopK ? 4 : 1) single_kernel(FusedParams P) {
  __shared__ __align__(16) uint8_t rec_smem[MODE == kTopK ? kWarps * kTopkMaxRec : 16];
  __shared__ __align__(8) uint64_t mbar[2];
  extern __shared__ __align__(128) uint8_t dsm[];
  const T* g = reinterpret_cast<const T*>(P.grad);
  const ChunkSrc<T> gsrc{g, P.pred, P.ef, 0};
  const float* pp = P.q.use_pred ? P.pred : nullptr;
  const float* pe = P.q.use_ef ? P.ef : nullptr;
  if constexpr (!kPrefetch<MODE, false>) {
    for (int ch = blockIdx.x; ch < P.nchunks; ch += gridDim.x) single_chunk<MODE, T, kOpt>(P, gsrc, ch, rec_smem);
    return;
  }
  ChunkPipe<T> pipe{mbar, dsm};
  pipe.init();
  const int c0 = blockIdx.x;
  if (c0 < P.nchunks && ChunkPipe<T>::full(P.n, c0)) pipe.issue(g, pp, pe, c0, 0);
  int it = 0;
  for (int ch = c0; ch < P.nchunks; ch += gridDim.x, ++it) {
    const int b = it & 1;
    const int cn = ch + gridDim.x;
    if (cn < P.nchunks && ChunkPipe<T>::full(P.n, cn)) pipe.issue(g, pp, pe, cn, b ^ 1);
    if (ChunkPipe<T>::full(P.n, ch)) {
      if (!pipe.wait(b, P.timeout_ns)) {
        if (threadIdx.x == 0) set_status(P.status, kTimeoutCopy, ch, 0);
        pipe.drain(P.timeout_ns);
        return;
      }
      single_chunk<MODE, T, kOpt>(P, pipe.buffer_source(b, ch), ch, rec_smem);
    } else {
      single_chunk<MODE, T, kOpt>(P, gsrc, ch, rec_smem);
    }
    __syncthreads();  // buffer b is reused two iterations on
  }
}

// ------------------------------------------ single-GPU building-block kernels
// Encode one rank's wire payload into a local buffer (oracle comparisons
// and multi-rank emulation on one GPU).
template <int MODE, typename T>
__global__ void __launch_bounds__(kThreads) encode_kernel(const T* g, const float* pred, const float* ef_in,
                                                          float* ef_out, int64_t n, int nblk, int nchunks, int k,
                                                          int rec_bytes, int chunk_bytes, QParams qp, uint8_t* out) {
  __shared__ __align__(16) uint8_t rec[Smem<MODE>::kRec];
  // ef_in and ef_out may differ here: copy-through by encoding from ef_in and
  // storing into ef_out (the fused kernels update in place).
  for (int c = blockIdx.x; c < nchunks; c += gridDim.x) {
    if (ef_in != ef_out && ef_in != nullptr) {
      // The encoders read EF through `ef` and write through the same pointer;
      // stage the chunk's EF into ef_out first so the in-place path applies.
      const int64_t e0 = (int64_t)c * kChunkBlocks * kBlock;
      const int64_t e1 = min64(n, e0 + (int64_t)kChunkBlocks * kBlock);
      for (int64_t i = e0 + threadIdx.x; i < e1; i += blockDim.x) ef_out[i] = ef_in[i];
      __syncthreads();
    }
    encode_chunk<MODE, T>(ChunkSrc<T>{g, pred, ef_out, 0}, ef_out, n, nblk, nchunks, k, rec_bytes, qp, c, rec);
    copy_record(out + (int64_t)c * chunk_bytes, rec, chunk_bytes);
    __syncthreads();
  }
}

template <int MODE, typename T>
__global__ void __launch_bounds__(kThreads) reduce_kernel(ReduceSrcs srcs, int world, T* out, float* pred, int64_t n,
                                                          int nblk, int nchunks, int k, int rec_bytes,
                                                          int chunk_bytes, FParams fp) {
  __shared__ __align__(16) uint8_t stage[Smem<MODE>::kStage];
  __shared__ __align__(16) float acc_smem[Smem<MODE>::kAcc];
  for (int c = blockIdx.x; c < nchunks; c += gridDim.x) {
    auto rc = [&](int src) { return srcs.p[src] + (int64_t)c * chunk_bytes; };
    decode_chunk<MODE, T, false>(rc, world, out, pred, n, nblk, nchunks, k, rec_bytes, fp, c, stage, acc_smem);
  }
}

// ------------------------------------------------------------- launchers
#define NGL_DISPATCH(MODE, DT, ...)                                               \
  [&] {                                                                           \
    if ((DT) == kF32) {                                                           \
      using T = float;                                                            \
      if ((MODE) == kInt4) { constexpr int M = kInt4; __VA_ARGS__(); }            \
      else if ((MODE) == kInt8) { constexpr int M = kInt8; __VA_ARGS__(); }       \
      else { constexpr int M = kTopK; __VA_ARGS__(); }                            \
    } else {                                                                      \
      using T = __nv_bfloat16;                                                    \
      if ((MODE) == kInt4) { constexpr int M = kInt4; __VA_ARGS__(); }            \
      else if ((MODE) == kInt8) { constexpr int M = kInt8; __VA_ARGS__(); }       \
      else { constexpr int M = kTopK; __VA_ARGS__(); }                            \
    }                                                                             \
  }()

// Dynamic shared memory of the prefetch pipeline; set on first use of each
// kernel instance (above the 48 KB default).
template <auto Kernel>
int prepare_dsmem(int bytes) {
  static bool done = false;  // one flag per kernel instance
  if (!done) {
    cudaFuncSetAttribute(Kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    done = true;
  }
  return bytes;
}

// ------------------------------------------------ prefetch pipeline check
// Every whole chunk of src goes through the ChunkPipe buffers (g slice only)
// and is written back to dst; the partial tail is copied directly.
__global__ void __launch_bounds__(kThreads) pipe_copy_kernel(const float* src, float* dst, int64_t n, int nchunks,
                                                             int vec, int* status) {
  __shared__ __align__(8) uint64_t mbar[2];
  extern __shared__ __align__(128) uint8_t dsm[];
  ChunkPipe<float> pipe{mbar, dsm};
  pipe.init();
  const int c0 = blockIdx.x;
  if (c0 < nchunks && ChunkPipe<float>::full(n, c0)) pipe.issue(src, nullptr, nullptr, c0, 0);
  int it = 0;
  for (int c = c0; c < nchunks; c += gridDim.x, ++it) {
    const int b = it & 1;
    const int cn = c + gridDim.x;
    if (cn < nchunks && ChunkPipe<float>::full(n, cn)) pipe.issue(src, nullptr, nullptr, cn, b ^ 1);
    const int64_t e0 = (int64_t)c * kChunkElems;
    if (ChunkPipe<float>::full(n, c)) {
      if (!pipe.wait(b, 1000000000ull)) {
        if (threadIdx.x == 0) set_status(status, kTimeoutCopy, c, 0);
        pipe.drain(1000000000ull);
        return;
      }
      const ChunkSrc<float> s = pipe.buffer_source(b, c);
      if (vec) {  // the encoders' read path: 8 elements per lane, vector loads
        float v[8];
        const int64_t l0 = (int64_t)threadIdx.x * 8;
        load8<float>(s.g, e0 + l0 - s.roff, 8, true, v);
        store8<float>(dst, e0 + l0, 8, true, v);
      } else {
        for (int i = threadIdx.x; i < kChunkElems; i += blockDim.x) dst[e0 + i] = s.g[e0 + i - s.roff];
      }
    } else {
      for (int64_t i = e0 + threadIdx.x; i < n; i += blockDim.x) dst[i] = src[i];
    }
    __syncthreads();
  }
}

cudaError_t launch_pipe_copy(const float* src, float* dst, int64_t n, int grid, int vec, int* status,
                             cudaStream_t stream) {
  const int nchunks = (int)((n + kChunkElems - 1) / kChunkElems);
  if (nchunks == 0) return cudaSuccess;
  const int dyn = prepare_dsmem<pipe_copy_kernel>(ChunkPipe<float>::kBytes);
  pipe_copy_kernel<<<grid, kThreads, dyn, stream>>>(src, dst, n, nchunks, vec, status);
  return cudaGetLastError();
}

// Dynamic shared memory of a kernel: the pipeline buffers when it prefetches.
template <int M, typename T, bool kExchange>
constexpr int dsmem_of() {
  return kPrefetch<M, kExchange> ? ChunkPipe<T>::kBytes : 0;
}

// Kernel instances.  Two-shot exists for the dense modes only, and the
// fused optimizer for fp32 dense buckets only; these helpers keep the other
// instances from being referenced (discarded branches inside a template).
template <int M, typename T, bool kOpt>
constexpr bool kHasOpt = !kOpt || (M != kTopK && sizeof(T) == 4);

template <int M, typename T, bool kOpt>
int occupancy_of(int variant) {
  int v = 1;
  if constexpr (kHasOpt<M, T, kOpt>) {
    if (variant == kVariantTwoShot) {
      if constexpr (M != kTopK)
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&v, twoshot_kernel<M, T, kOpt>, kThreads, dsmem_of<M, T, true>());
    } else if (variant == kVariantOneShot) {
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&v, oneshot_kernel<M, T, kOpt>, kThreads, dsmem_of<M, T, true>());
    } else {
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(
          &v, single_kernel<M, T, kOpt>, kThreads,
          prepare_dsmem<single_kernel<M, T, kOpt>>(dsmem_of<M, T, false>()));
    }
  }
  return v;
}

template <int M, typename T, bool kOpt>
void launch_instance(const FusedParams& P, int variant, int grid, cudaStream_t stream) {
  if constexpr (kHasOpt<M, T, kOpt>) {
    if (variant == kVariantSingle) {
      const int dyn = prepare_dsmem<single_kernel<M, T, kOpt>>(dsmem_of<M, T, false>());
      single_kernel<M, T, kOpt><<<grid, kThreads, dyn, stream>>>(P);
    } else if (variant == kVariantTwoShot) {
      if constexpr (M != kTopK) twoshot_kernel<M, T, kOpt><<<grid, kThreads, dsmem_of<M, T, true>(), stream>>>(P);
    } else {
      oneshot_kernel<M, T, kOpt><<<grid, kThreads, dsmem_of<M, T, true>(), stream>>>(P);
    }
  }
}

int fused_grid(int nchunks, int mode, int dtype, int variant, int cap, int device, int opt) {
  static int occ_cache[2][3][2][3] = {};
  static int sms = 0;
  if (sms == 0) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  opt = (opt && dtype == kF32 && mode != kTopK) ? 1 : 0;
  int& occ = occ_cache[opt][variant][dtype][mode];
  if (occ == 0) {
    int v = 1;
    NGL_DISPATCH(mode, dtype, [&] { v = opt ? occupancy_of<M, T, true>(variant) : occupancy_of<M, T, false>(variant); });
    occ = v > 0 ? v : 1;
  }
  int g = occ * sms;
  if (variant == kVariantSingle) {
    g = 4 * sms;
    const int need = nchunks;  // one chunk = kWarps blocks = one CTA iteration
    return need < g ? (need > 0 ? need : 1) : g;
  }
  if (cap > 0 && cap < g) g = cap;
  if (g > kMaxCols) g = kMaxCols;
  if (nchunks < g) g = nchunks;
  return g > 0 ? g : 1;
}

cudaError_t launch_fused(const FusedParams& P, int mode, int dtype, int variant, int grid, cudaStream_t stream) {
  const bool opt = P.f.opt.segs != nullptr;
  if (opt && (dtype != kF32 || mode == kTopK)) return cudaErrorInvalidValue;
  NGL_DISPATCH(mode, dtype, [&] {
    if (opt) launch_instance<M, T, true>(P, variant, grid, stream);
    else launch_instance<M, T, false>(P, variant, grid, stream);
  });
  return cudaGetLastError();
}

cudaError_t launch_encode(const void* g, const float* pred, const float* ef_in, float* ef_out, int64_t n, int k,
                          const QParams& qp, uint8_t* out, int mode, int dtype, int grid, cudaStream_t stream) {
  const int nblk = (int)((n + kBlock - 1) / kBlock);
  const int nchunks = (nblk + kChunkBlocks - 1) / kChunkBlocks;
  const int rec = topk_record_bytes(k);
  const int cb = chunk_record_bytes(mode, k);
  NGL_DISPATCH(mode, dtype, [&] {
    encode_kernel<M, T><<<grid, kThreads, 0, stream>>>(reinterpret_cast<const T*>(g), pred, ef_in, ef_out, n, nblk,
                                                      nchunks, k, rec, cb, qp, out);
  });
  return cudaGetLastError();
}

cudaError_t launch_reduce(const ReduceSrcs& srcs, int world, void* out, float* pred, int64_t n, int k,
                          const FParams& fp, int mode, int dtype, int grid, cudaStream_t stream) {
  const int nblk = (int)((n + kBlock - 1) / kBlock);
  const int nchunks = (nblk + kChunkBlocks - 1) / kChunkBlocks;
  const int rec = topk_record_bytes(k);
  const int cb = chunk_record_bytes(mode, k);
  NGL_DISPATCH(mode, dtype, [&] {
    reduce_kernel<M, T><<<grid, kThreads, 0, stream>>>(srcs, world, reinterpret_cast<T*>(out), pred, n, nblk,
                                                      nchunks, k, rec, cb, fp);
  });
  return cudaGetLastError();
}

}  // namespace dev
}  // namespace ngl
