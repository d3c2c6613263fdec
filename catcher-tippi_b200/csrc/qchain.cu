// Persistent executor of a chain of small-M affine INT8 linears (the batch-1
// streaming chunk: M = lookahead + 1 <= 16 rows, every linear of the 24
// FastConformer blocks in sequence).  Replaces one K1 launch per linear
// (QuantizedLinear::forward_array, crates/nemotron-mlx/src/model/
// layers.rs:298-310, called once per linear by the encoder blocks,
// encoder.rs) by one cooperative launch for the whole chain.
//
// Why: at M = 14 a linear is a few MB of weights; streamed at HBM speed it
// takes well under a microsecond, while a dependent kernel launch costs
// several.  Weights do not depend on activations, so each CTA streams the
// weight tiles of its share of ALL steps through a ring of shared-memory
// slots (TMA, L2 evict-first) as far ahead as the ring allows, and only the
// short activation-dependent part of each step waits for its producers.
//
// Work decomposition.  Step s is cut into items (16*rt weight rows) x (a
// K-range of sb_per_item 64-wide sub-blocks) x (one 16-token tile); items of
// all steps are numbered in step order and CTA c takes items c, c + grid,
// c + 2*grid, ...  Every CTA therefore meets the steps in order, and a step's
// items only wait for earlier steps: with all CTAs resident (cooperative
// launch) the schedule cannot deadlock.
//
// Per item (8 consumer warps; a ninth warp issues the weight copies):
//   scales/biases -> registers (before any wait), producer-completion wait,
//   activation loads, exact f16 MMAs on 1024 + q (gemv_core.cuh), reduction
//   over warps, then either the output epilogue, or (K split over items) an
//   f32 partial in global memory and an arrival count; the last arriving item
//   of a (band, token tile) sums the partials in slice order (deterministic)
//   and finishes it.  A finished unit bumps the step's completion counter.
// Every wait is bounded (kWaitLimitNs): on timeout the CTA sets the status
// word and an abort flag that releases every other waiter.
#include "common.cuh"
#include "gemv_core.cuh"
#include "qchain.hpp"

namespace cq {

namespace {

constexpr int kCW = 8;                    // consumer warps
constexpr int kCThreads = kCW * 32;       // consumer threads (named barrier 1)
constexpr int kThreads = kCThreads + 32;  // + producer warp
constexpr int kSlots = 5;
constexpr int kMaxRB = 32;
constexpr int kMaxSb = 16;                      // sub-blocks per item
constexpr int kSbPerWarp = kMaxSb / kCW;        // two
// (s, b) pairs per item: RB * sbn * SUBG <= kChainSlotBytes / 64 * 2
constexpr int kMaxPairs = kChainSlotBytes / 64 * 2;
constexpr int kMaxScalePerThread = kMaxPairs / kCThreads;

// Raw T group scales, group biases and output biases of one item, staged by
// the producer warp next to the item's weight tile.
struct ScaleStage {
  uint16_t s[kMaxPairs];
  uint16_t b[kMaxPairs];
  uint16_t bias[kMaxRB];
};

struct ChainSmem {
  static constexpr size_t slots = 0;
  static constexpr size_t stage = slots + static_cast<size_t>(kSlots) * kChainSlotBytes;
  static constexpr size_t sbsm = stage + static_cast<size_t>(kSlots) * sizeof(ScaleStage);
  static constexpr size_t red = sbsm + static_cast<size_t>(kMaxPairs) * sizeof(float2);
  static constexpr size_t bars = red + static_cast<size_t>(kCW) * kMaxRB * 16 * sizeof(float);
  static constexpr size_t flags = bars + 2 * kSlots * sizeof(uint64_t);
  static constexpr size_t total = flags + 16 * sizeof(int);
};

__device__ __forceinline__ void consumer_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kCThreads) : "memory");
}

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ int ld_volatile_i32(const int* p) {
  return *reinterpret_cast<const volatile int*>(p);
}

__device__ __forceinline__ float ld_cg_f32(const float* p) {
  float v;
  asm volatile("ld.global.cg.f32 %0, [%1];" : "=f"(v) : "l"(p));
  return v;
}

// Completion count with release semantics: the outputs this CTA stored before
// the consumer barrier are visible to whoever observes the new count.
__device__ __forceinline__ void red_release_add(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// K-split arrival: returns the previous count, wrapping to 0 at `wrap`.
__device__ __forceinline__ unsigned atom_inc_acq_rel(unsigned* p, unsigned wrap) {
  unsigned old;
  asm volatile("atom.acq_rel.gpu.global.inc.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(wrap) : "memory");
  return old;
}

__device__ void raise_abort(const ChainArgs& a) {
  if (a.status != nullptr) atomicOr(a.status, kStatusWaitTimeout);
  atomicExch(a.abort_flag, 1);
}

// mbarrier phase wait bounded in time and released early by an abort.
__device__ bool slot_wait(uint64_t* bar, uint32_t parity, const ChainArgs& a) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (ld_volatile_i32(a.abort_flag) != 0) return false;
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      raise_abort(a);
      return false;
    }
  }
}

// Thread 0 of the consumers: every producer step of `st` has completed.
__device__ bool deps_wait(const ChainArgs& a, const ChainStep& st) {
#pragma unroll 1
  for (int d = 0; d < kChainMaxDeps; ++d) {
    const int p = st.dep[d];
    if (p < 0) continue;
    const unsigned target = static_cast<unsigned>(a.steps[p].units);
    if (ld_acquire_u32(a.done + p) >= target) continue;
    // Every CTA polls the counter its producers increment: back off between
    // polls so that the increments are not starved at the L2 slice.
    const uint64_t t0 = globaltimer_ns();
    unsigned polls = 0;
    while (ld_acquire_u32(a.done + p) < target) {
      if (ld_volatile_i32(a.abort_flag) != 0) return false;
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        raise_abort(a);
        return false;
      }
      if (++polls > 4) __nanosleep(64);
    }
  }
  // the acquire loads order this thread's later accesses; the consumer
  // barrier that follows orders the other threads'
  return true;
}

template <int DT>
__device__ __forceinline__ float bits_to_float(uint16_t v) {
  if constexpr (DT == kBF16) return __uint_as_float(static_cast<uint32_t>(v) << 16);
  else return __half2float(__ushort_as_half(v));
}

template <int DT>
__device__ __forceinline__ uint32_t float_to_bits(float v) {
  if constexpr (DT == kBF16) return __bfloat16_as_ushort(__float2bfloat16_rn(v));
  else return __half_as_ushort(__float2half_rn(v));
}

__device__ __forceinline__ void st_tagged(unsigned long long* p, uint32_t lo, uint32_t tag) {
  const unsigned long long w = (static_cast<unsigned long long>(tag) << 32) | lo;
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}

__device__ __forceinline__ void ld_tagged_x2(const unsigned long long* p, unsigned long long& a,
                                             unsigned long long& b) {
  asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

// This lane's 16 activation values of token m for one 64-wide sub-block (the
// layout of load_x_raw), read from the producer's tagged copy; spins until
// every word carries `tag`.  Returns false on timeout or abort.
template <int G>
__device__ bool load_x_tagged(const ChainStep& st, const ChainArgs& a, int m, int kb, int c,
                              uint32_t tag, uint4& r0, uint4& r1) {
  r0 = make_uint4(0, 0, 0, 0);
  r1 = make_uint4(0, 0, 0, 0);
  if (m >= st.M) return true;
  const unsigned long long* row = st.x_tagged + static_cast<size_t>(m) * st.x_tagged_ld + st.x_tagged_col;
  // word runs (4 words = 8 values each): G >= 64: kb + 16c + [0, 16);
  // G == 32: kb + 8c + [0, 8) and kb + 32 + 8c + [0, 8)
  const int w0 = (G >= 64) ? (kb + 16 * c) / 2 : (kb + 8 * c) / 2;
  const int w1 = (G >= 64) ? w0 + 4 : (kb + 32 + 8 * c) / 2;
  const bool second = (G >= 64) || (kb + 32 < st.K);
  uint64_t t0 = 0;
  unsigned polls = 0;
  while (true) {
    unsigned long long v[8];
    ld_tagged_x2(row + w0, v[0], v[1]);
    ld_tagged_x2(row + w0 + 2, v[2], v[3]);
    if (second) {
      ld_tagged_x2(row + w1, v[4], v[5]);
      ld_tagged_x2(row + w1 + 2, v[6], v[7]);
    } else {
      v[4] = v[5] = v[6] = v[7] = static_cast<unsigned long long>(tag) << 32;
    }
    bool ready = true;
#pragma unroll
    for (int i = 0; i < 8; ++i) ready = ready && static_cast<uint32_t>(v[i] >> 32) == tag;
    if (ready) {
      r0 = make_uint4(static_cast<uint32_t>(v[0]), static_cast<uint32_t>(v[1]),
                      static_cast<uint32_t>(v[2]), static_cast<uint32_t>(v[3]));
      if (second)
        r1 = make_uint4(static_cast<uint32_t>(v[4]), static_cast<uint32_t>(v[5]),
                        static_cast<uint32_t>(v[6]), static_cast<uint32_t>(v[7]));
      return true;
    }
    if (polls == 0) t0 = globaltimer_ns();
    if (++polls > 2) __nanosleep(64);
    if ((polls & 15) == 0) {
      if (ld_volatile_i32(a.abort_flag) != 0) return false;
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        raise_abort(a);
        return false;
      }
    }
  }
}

// One profile stamp of item t (thread 0 / producer lane only).
__device__ __forceinline__ void stamp(const ChainArgs& a, int t, int k) {
  if (a.trace != nullptr) a.trace[static_cast<size_t>(t) * kChainTraceStamps + k] = globaltimer_ns();
}

struct ItemPos {
  int ks, band, mt, unit, n0, sb0, sbn;
};

__device__ __forceinline__ ItemPos decode_item(const ChainStep& st, int u) {
  ItemPos p;
  p.ks = u % st.kslices;
  const int rest = u / st.kslices;
  p.band = rest % st.bands;
  p.mt = rest / st.bands;
  p.unit = p.mt * st.bands + p.band;
  p.n0 = p.band * 16 * st.rt;
  const int nsb = (st.K + 63) >> 6;
  p.sb0 = p.ks * st.sb_per_item;
  p.sbn = max(0, min(st.sb_per_item, nsb - p.sb0));
  return p;
}

// One item on the consumer warps.  Returns false if the chain was aborted.
template <int DT, int G, int RT>
__device__ bool run_item(const ChainArgs& a, const ChainStep& st, int s, int t, const ItemPos& p,
                         const uint8_t* slot, const ScaleStage* stage, uint64_t* full,
                         uint32_t full_parity, uint64_t* empty, bool need_deps, uint32_t tag,
                         uint8_t* smem) {
  constexpr int RB = 16 * RT;
  constexpr int SUBG = (G == 32) ? 2 : 1;
  float2* sbsm = reinterpret_cast<float2*>(smem + ChainSmem::sbsm);
  float* red = reinterpret_cast<float*>(smem + ChainSmem::red);
  int* flags = reinterpret_cast<int*>(smem + ChainSmem::flags);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int c = lane & 3, r4 = lane >> 2;
  if (tid == 0) stamp(a, t, 1);

  // ---- producers of this step's activations
  if (need_deps) {
    if (tid == 0) {
      flags[0] = deps_wait(a, st) ? 1 : 0;
      stamp(a, t, 2);
    }
    consumer_sync();
    if (flags[0] == 0) return false;
  }

  // ---- activations: every load of this warp's sub-blocks in flight at once
  uint4 xr[kSbPerWarp][2][2];
  if (st.x_tagged != nullptr) {
    bool ok = true;
#pragma unroll
    for (int u = 0; u < kSbPerWarp; ++u) {
      const int j = warp + u * kCW;
      if (j < p.sbn) {
        const int kb = (p.sb0 + j) * 64;
        ok = ok && load_x_tagged<G>(st, a, p.mt * 16 + r4, kb, c, tag, xr[u][0][0], xr[u][0][1]);
        ok = ok && load_x_tagged<G>(st, a, p.mt * 16 + 8 + r4, kb, c, tag, xr[u][1][0], xr[u][1][1]);
      }
    }
    if (!ok) flags[6] = 1;  // any thread: the chain was aborted
  } else {
#pragma unroll
    for (int u = 0; u < kSbPerWarp; ++u) {
      const int j = warp + u * kCW;
      if (j < p.sbn) {
        const int kb = (p.sb0 + j) * 64;
        load_x_raw<G>(st.x, st.ldx, st.M, st.K, p.mt * 16 + r4, kb, c, xr[u][0][0], xr[u][0][1]);
        load_x_raw<G>(st.x, st.ldx, st.M, st.K, p.mt * 16 + 8 + r4, kb, c, xr[u][1][0],
                      xr[u][1][1]);
      }
    }
  }
  // the weight tile and staged scales of this item (thread 0 waits, bounded;
  // everyone then observes the completed phase itself)
  if (tid == 0) {
    flags[1] = slot_wait(full, full_parity, a) ? 1 : 0;
    stamp(a, t, 3);
  }
  consumer_sync();
  if (flags[1] == 0 || flags[6] != 0) return false;
#pragma unroll 1
  for (int i = 0; i < 64 && !mbar_try_wait(full, full_parity); ++i) {
  }
  // (s, b - 1024 s) in fp32 for the MMA epilogue, [jh][row] order as staged
  const int total = p.sbn * SUBG * RB;
#pragma unroll
  for (int i = 0; i < kMaxScalePerThread; ++i) {
    const int e = tid + i * kCThreads;
    if (e < total) {
      const float sv = bits_to_float<DT>(stage->s[e]);
      const float bv = bits_to_float<DT>(stage->b[e]);
      sbsm[e] = make_float2(sv, fmaf(-1024.0f, sv, bv));
    }
  }
  consumer_sync();

  float acc[RT][2][4];
#pragma unroll
  for (int i = 0; i < RT; ++i)
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[i][nt][e] = 0.f;
#pragma unroll
  for (int u = 0; u < kSbPerWarp; ++u) {
    const int j = warp + u * kCW;
    if (j >= p.sbn) break;
    const XOperands<G> xo = x_operands<DT, G>(xr[u], lane);
    subblock_mma<DT, G, RT>(slot + static_cast<size_t>(j) * RB * 64,
                            sbsm + static_cast<size_t>(j) * SUBG * RB, xo, lane, acc);
  }

  // ---- reduce over warps; the slot is free once every warp is past it
#pragma unroll
  for (int i = 0; i < RT; ++i) {
    const int ra = 16 * i + r4, rb = ra + 8;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      *reinterpret_cast<float2*>(&red[(warp * RB + ra) * 16 + 8 * nt + 2 * c]) =
          make_float2(acc[i][nt][0], acc[i][nt][1]);
      *reinterpret_cast<float2*>(&red[(warp * RB + rb) * 16 + 8 * nt + 2 * c]) =
          make_float2(acc[i][nt][2], acc[i][nt][3]);
    }
  }
  consumer_sync();
  if (tid == 0) {
    mbar_arrive(empty);
    stamp(a, t, 4);
  }

  const bool has_bias = st.bias != nullptr;
  bool finished = false;
  // Output pairs (rows 2r, 2r + 1 of the band) of one token: consecutive
  // threads take consecutive pairs; each pair is stored to y and, when a
  // later step reads it, as one tagged word.
  auto emit = [&](int r2, int tok, float v0, float v1) {
    const int n = p.n0 + 2 * r2, m = p.mt * 16 + tok;
    if (m >= st.M || n >= st.N) return;
    const float o0 = epilogue_value<DT>(v0, has_bias, bits_to_float<DT>(stage->bias[2 * r2]), st.act);
    st_t<DT>(st.y, static_cast<size_t>(m) * st.ldy + n, o0);
    float o1 = 0.f;
    if (n + 1 < st.N) {
      o1 = epilogue_value<DT>(v1, has_bias, bits_to_float<DT>(stage->bias[2 * r2 + 1]), st.act);
      st_t<DT>(st.y, static_cast<size_t>(m) * st.ldy + n + 1, o1);
    }
    if (st.y_tagged != nullptr)
      st_tagged(st.y_tagged + static_cast<size_t>(m) * st.y_tagged_ld + n / 2,
                float_to_bits<DT>(o0) | (n + 1 < st.N ? float_to_bits<DT>(o1) << 16 : 0u), tag);
  };
  if (st.kslices == 1) {
    for (int e = tid; e < RB * 8; e += kCThreads) {
      const int r2 = e % (RB / 2), tok = e / (RB / 2);
      float v0 = 0.f, v1 = 0.f;
#pragma unroll
      for (int w = 0; w < kCW; ++w) {
        v0 += red[(w * RB + 2 * r2) * 16 + tok];
        v1 += red[(w * RB + 2 * r2 + 1) * 16 + tok];
      }
      emit(r2, tok, v0, v1);
    }
    finished = true;
  } else {
    float* part = st.partial + (static_cast<size_t>(p.unit) * st.kslices + p.ks) * RB * 16;
    for (int e = tid; e < RB * 16; e += kCThreads) {
      float v = 0.f;
#pragma unroll
      for (int w = 0; w < kCW; ++w) v += red[w * RB * 16 + e];
      part[e] = v;
    }
    consumer_sync();
    if (tid == 0) {
      const unsigned old = atom_inc_acq_rel(st.arrive + p.unit, static_cast<unsigned>(st.kslices - 1));
      flags[2] = old == static_cast<unsigned>(st.kslices - 1) ? 1 : 0;
    }
    consumer_sync();
    if (flags[2] != 0) {
      // last slice of this (band, token tile): sum the partials in slice order
      const float* base = st.partial + static_cast<size_t>(p.unit) * st.kslices * RB * 16;
      for (int e = tid; e < RB * 8; e += kCThreads) {
        const int r2 = e % (RB / 2), tok = e / (RB / 2);
        float v0 = 0.f, v1 = 0.f;
        for (int q = 0; q < st.kslices; ++q) {
          const float* pq = base + static_cast<size_t>(q) * RB * 16;
          v0 += ld_cg_f32(pq + (2 * r2) * 16 + tok);
          v1 += ld_cg_f32(pq + (2 * r2 + 1) * 16 + tok);
        }
        emit(r2, tok, v0, v1);
      }
      finished = true;
    }
  }
  consumer_sync();  // red, sbsm and the outputs of this item are settled
  // the count only matters to steps that wait for it; a release RMW stalls
  // until this CTA's stores are performed, so it is skipped otherwise
  if (finished && tid == 0 && st.signal) red_release_add(a.done + s, 1u);
  if (tid == 0) stamp(a, t, 5);
  return true;
}

template <int DT, int G>
__global__ void __launch_bounds__(kThreads, 1) qchain_kernel(const ChainArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* slots = smem + ChainSmem::slots;
  ScaleStage* stage = reinterpret_cast<ScaleStage*>(smem + ChainSmem::stage);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + ChainSmem::bars);
  uint64_t* empty = full + kSlots;
  int* flags = reinterpret_cast<int*>(smem + ChainSmem::flags);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int grid = gridDim.x;

  if (tid == 0) {
    for (int i = 0; i < kSlots; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    fence_mbar_init();
    flags[3] = 0;  // items whose copies were issued
    flags[4] = 0;  // items consumed
    flags[6] = 0;  // a tagged load gave up
    unsigned tag = *reinterpret_cast<volatile unsigned*>(a.epoch) + 1u;
    if (tag == 0) tag = 1;  // zero-filled words never carry a live tag
    flags[7] = static_cast<int>(tag);
  }
  __syncthreads();
  const uint32_t tag = static_cast<uint32_t>(flags[7]);

  if (warp == kCW) {
    // ---- producer: weight tiles and scales of this CTA's items, as far
    // ahead as the ring allows
    const uint64_t pol_once = l2_policy_evict_first();
    const uint64_t pol_keep = l2_policy_evict_normal();
    int s = 0, i = 0;
#pragma unroll 1
    for (int t = blockIdx.x; t < a.total_items; t += grid, ++i) {
      while (t >= a.steps[s].item_base + a.steps[s].items) ++s;
      const ChainStep& st = a.steps[s];
      const int slot = i % kSlots;
      int go = 1;
      if (lane == 0 && i >= kSlots) go = slot_wait(&empty[slot], ((i / kSlots) - 1) & 1, a) ? 1 : 0;
      if (__shfl_sync(0xFFFFFFFFu, go, 0) == 0) break;
      const ItemPos p = decode_item(st, t - st.item_base);
      const int rb = 16 * st.rt;
      ScaleStage* sg = stage + slot;
      // scales/biases in [jh][row] order (jh: group slot within the item)
      const int subg = (G == 32) ? 2 : 1;
      const int per_row = p.sbn * subg;
      const int total = per_row * rb;
      const int gpr = st.K / G;
      const uint16_t* sc = static_cast<const uint16_t*>(st.scales);
      const uint16_t* bi = static_cast<const uint16_t*>(st.biases);
      for (int e = lane; e < total; e += 32) {
        const int jh = e / rb, row = e - jh * rb;
        const int n = p.n0 + row;
        const int kfirst = (p.sb0 + jh / subg) * 64 + (jh % subg) * 32;
        uint16_t sv = 0, bv = 0;
        if (n < st.N && kfirst < st.K) {
          const size_t gi = static_cast<size_t>(n) * gpr + kfirst / G;
          sv = __ldg(sc + gi);
          bv = __ldg(bi + gi);
        }
        sg->s[e] = sv;
        sg->b[e] = bv;
      }
      if (lane < rb)
        sg->bias[lane] = (st.bias != nullptr && p.n0 + lane < st.N)
                             ? __ldg(static_cast<const uint16_t*>(st.bias) + p.n0 + lane)
                             : static_cast<uint16_t>(0);
      __syncwarp();
      if (lane == 0) {
        uint8_t* dst = slots + static_cast<size_t>(slot) * kChainSlotBytes;
        const uint64_t pol = st.evict_first ? pol_once : pol_keep;
        mbar_arrive_expect_tx(&full[slot], static_cast<uint32_t>(p.sbn * rb * 64));
        for (int j = 0; j < p.sbn; ++j)
          tma_load_2d(dst + static_cast<size_t>(j) * rb * 64, st.wmap, (p.sb0 + j) * 64, p.n0,
                      &full[slot], pol);
        stamp(a, t, 0);
        flags[3] = i + 1;
      }
    }
    __syncwarp();
  } else {
    // ---- consumers
    int s = 0, i = 0, deps_ok = -1;
#pragma unroll 1
    for (int t = blockIdx.x; t < a.total_items; t += grid, ++i) {
      while (t >= a.steps[s].item_base + a.steps[s].items) ++s;
      const ChainStep& st = a.steps[s];
      const ItemPos p = decode_item(st, t - st.item_base);
      const int slot = i % kSlots;
      const uint8_t* src = slots + static_cast<size_t>(slot) * kChainSlotBytes;
      const uint32_t parity = (i / kSlots) & 1;
      const bool need = deps_ok != s;
      const bool ok = st.rt == 1
          ? run_item<DT, G, 1>(a, st, s, t, p, src, stage + slot, &full[slot], parity,
                               &empty[slot], need, tag, smem)
          : run_item<DT, G, 2>(a, st, s, t, p, src, stage + slot, &full[slot], parity,
                               &empty[slot], need, tag, smem);
      if (!ok) break;
      deps_ok = s;
      if (tid == 0) flags[4] = i + 1;
    }
  }
  __syncthreads();

  if (tid == 0) {
    // after an abort: copies issued for items never consumed are waited for
    // (bounded) before the shared memory is released
    for (int i = flags[4]; i < flags[3]; ++i)
      mbar_wait_bounded(&full[i % kSlots], (i / kSlots) & 1, a.status);
    // the last CTA out resets the counters for the next launch
    __threadfence();
    const unsigned old = atomicInc(a.exit_count, static_cast<unsigned>(grid - 1));
    flags[5] = old == static_cast<unsigned>(grid - 1) ? 1 : 0;
    if (flags[5] != 0) __threadfence();
  }
  __syncthreads();
  if (flags[5] != 0) {
    for (int s = tid; s < a.nsteps; s += kThreads) a.done[s] = 0;
    for (int u = tid; u < a.narrive; u += kThreads) a.arrive[u] = 0;
    if (tid == 0) {
      *a.abort_flag = 0;
      *a.epoch = tag;  // the next launch tags with a new value
    }
  }
}

template <int DT>
cudaError_t launch_g(int group, const ChainArgs& a, int grid, cudaStream_t stream, bool set_only) {
  void (*kern)(const ChainArgs) = nullptr;
  switch (group) {
    case 32: kern = qchain_kernel<DT, 32>; break;
    case 64: kern = qchain_kernel<DT, 64>; break;
    case 128: kern = qchain_kernel<DT, 128>; break;
    default: return cudaErrorInvalidValue;
  }
  if (set_only)
    return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(ChainSmem::total));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = ChainSmem::total;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, a);
}

}  // namespace

size_t chain_smem_bytes() { return ChainSmem::total; }
int chain_threads() { return kThreads; }

cudaError_t chain_set_smem(int dtype, int group) {
  const ChainArgs none{};
  if (dtype == kF16) return launch_g<kF16>(group, none, 0, nullptr, true);
  if (dtype == kBF16) return launch_g<kBF16>(group, none, 0, nullptr, true);
  return cudaErrorInvalidValue;
}

cudaError_t launch_chain(int dtype, int group, const ChainArgs& args, int grid,
                         cudaStream_t stream) {
  if (dtype == kF16) return launch_g<kF16>(group, args, grid, stream, false);
  if (dtype == kBF16) return launch_g<kBF16>(group, args, grid, stream, false);
  return cudaErrorInvalidValue;
}

}  // namespace cq
