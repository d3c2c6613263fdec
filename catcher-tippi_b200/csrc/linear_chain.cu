// Host side of the persistent linear-chain executor (linear_chain.hpp): step
// validation, buffer-derived dependencies, the per-step work decomposition
// and the device-resident step table.
#include "linear_chain.hpp"

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>

namespace nemotron_cuda {

namespace {

struct ByteRange {
  uintptr_t lo, hi;  // [lo, hi)
  bool overlaps(const ByteRange& o) const { return lo < o.hi && o.lo < hi; }
};

ByteRange range_of(const void* p, int ld, int rows, int cols, size_t elem) {
  const uintptr_t lo = reinterpret_cast<uintptr_t>(p);
  return ByteRange{lo, lo + (static_cast<size_t>(rows - 1) * ld + cols) * elem};
}

struct StepPlan {
  int rt, spi, kslices, items;
};

// Fewest rounds of items over the grid first (each round is a serial item per
// CTA on the step's critical path), then the fewest K slices (a split adds a
// partial-sum round trip), then the smallest item.
StepPlan plan_step(int N, int K, int M, int grid) {
  const int nsb = (K + 63) / 64;
  const int mtiles = (M + 15) / 16;
  int force_rt = 0, force_spi = 0;
  if (const char* env = std::getenv("CQ_CHAIN_PLAN"))
    if (std::sscanf(env, "%d,%d", &force_rt, &force_spi) != 2) force_rt = force_spi = 0;
  StepPlan best{0, 0, 0, 0};
  long best_key = -1;
  for (int rt : {1, 2}) {
    for (int spi : {16, 8, 4, 2, 1}) {
      if (16 * rt * spi * 64 > cq::kChainSlotBytes) continue;
      if (force_rt != 0 && (rt != force_rt || spi != force_spi)) continue;
      const int s = std::min(spi, nsb);
      const int ks = (nsb + s - 1) / s;
      const int bands = (N + 16 * rt - 1) / (16 * rt);
      const int items = bands * ks * mtiles;
      const int rounds = (items + grid - 1) / grid;
      const long key = (static_cast<long>(rounds) << 40) | (static_cast<long>(ks) << 20) | (rt * s);
      if (best_key < 0 || key < best_key) {
        best_key = key;
        best = StepPlan{rt, s, ks, items};
      }
    }
  }
  if (best_key < 0) throw_invalid("CQ_CHAIN_PLAN names no valid item shape");
  return best;
}

}  // namespace

LinearChain::LinearChain(const std::vector<ChainStepSpec>& specs) {
  if (specs.empty()) throw_invalid("a linear chain needs at least one step");
  const int n = static_cast<int>(specs.size());
  for (int i = 0; i < n; ++i) {
    const ChainStepSpec& s = specs[i];
    const std::string at = "chain step " + std::to_string(i) + ": ";
    if (s.layer == nullptr) throw_invalid(at + "layer must not be null");
    if (s.x == nullptr || s.y == nullptr) throw_invalid(at + "input and output must not be null");
    if (i == 0) {
      device_ = s.layer->device();
      dtype_ = s.layer->dtype();
      group_ = s.layer->group_size();
    }
    if (s.layer->device() != device_ || s.layer->dtype() != dtype_ || s.layer->group_size() != group_)
      throw_invalid(at + "every layer of a chain needs the same device, dtype and group size");
    if (dtype_ != CQ_F16 && dtype_ != CQ_BF16) throw_invalid(at + "chains run f16 or bf16 layers");
    if (s.rows < 1 || s.rows >= cq::kGemmMinRows)
      throw_invalid(at + "rows must be in [1, " + std::to_string(cq::kGemmMinRows) + ")");
    if (s.ldx < s.layer->input_dims() || s.ldy < s.layer->output_dims())
      throw_invalid(at + "leading dimensions are smaller than the layer");
    if ((reinterpret_cast<uintptr_t>(s.x) & 15) != 0 || (s.ldx % 8) != 0)
      throw_invalid(at + "input rows must be 16-byte aligned (x % 16 == 0 and ldx % 8 == 0)");
    if (s.act != CQ_ACT_NONE && s.act != CQ_ACT_SILU && s.act != CQ_ACT_RELU)
      throw_invalid(at + "unknown activation " + std::to_string(s.act));
  }

  DeviceContext& ctx = device_context(device_);
  DeviceGuard guard(device_);
  grid_ = ctx.num_sms;
  check_cuda(cq::chain_set_smem(dtype_, group_), "chain shared memory");

  // ---- dependencies: every conflicting earlier step, minus those another
  // conflicting step already waits for (directly or transitively)
  std::vector<std::vector<char>> anc(n, std::vector<char>(n, 0));
  std::vector<std::vector<int>> deps(n);
  std::vector<int> tagged_src(n, -1), tagged_col(n, 0);
  for (int i = 0; i < n; ++i) {
    const ChainStepSpec& s = specs[i];
    const ByteRange xi = range_of(s.x, s.ldx, s.rows, s.layer->input_dims(), 2);
    const ByteRange yi = range_of(s.y, s.ldy, s.rows, s.layer->output_dims(), 2);
    if (xi.overlaps(yi)) throw_invalid("chain step " + std::to_string(i) + ": input and output overlap");
    std::vector<int> conflicts, raw;
    std::vector<char> only_raw(i, 0);
    for (int j = 0; j < i; ++j) {
      const ChainStepSpec& t = specs[j];
      const ByteRange xj = range_of(t.x, t.ldx, t.rows, t.layer->input_dims(), 2);
      const ByteRange yj = range_of(t.y, t.ldy, t.rows, t.layer->output_dims(), 2);
      const bool r = yj.overlaps(xi), other = xj.overlaps(yi) || yj.overlaps(yi);
      if (r) raw.push_back(j);
      if (r || other) conflicts.push_back(j);
      only_raw[j] = r && !other;
    }
    // A single producer whose output rows line up with this step's input rows
    // is read through its tagged copy: no completion wait for it.
    tagged_src[i] = -1;
    if (raw.size() == 1 && only_raw[raw[0]]) {
      const int j = raw[0];
      const ChainStepSpec& t = specs[j];
      const intptr_t off = reinterpret_cast<intptr_t>(s.x) - reinterpret_cast<intptr_t>(t.y);
      const int col = static_cast<int>(off / 2);
      if (s.ldx == t.ldy && off >= 0 && off % 4 == 0 && off < static_cast<intptr_t>(t.ldy) * 2 &&
          t.ldy % 4 == 0 && s.rows <= t.rows &&
          col + s.layer->input_dims() <= t.layer->output_dims()) {
        tagged_src[i] = j;
        tagged_col[i] = col / 2;
        conflicts.erase(std::find(conflicts.begin(), conflicts.end(), j));
      }
    }
    for (int j : conflicts) {
      bool implied = false;
      for (int k : conflicts)
        if (k != j && anc[k][j]) implied = true;
      if (!implied) deps[i].push_back(j);
    }
    if (static_cast<int>(deps[i].size()) > cq::kChainMaxDeps)
      throw_invalid("chain step " + std::to_string(i) + " depends on more than " +
                    std::to_string(cq::kChainMaxDeps) + " unrelated earlier steps");
    for (int d : deps[i]) {
      anc[i][d] = 1;
      for (int k = 0; k < n; ++k)
        if (anc[d][k]) anc[i][k] = 1;
    }
  }

  // ---- work decomposition and device tables
  maps_ = DeviceBuffer(static_cast<size_t>(n) * sizeof(CUtensorMap));
  std::vector<CUtensorMap> maps(n);
  host_.resize(n);
  size_t partial_floats = 0, arrive_count = 0;
  std::vector<size_t> partial_off(n, 0), arrive_off(n, 0);
  for (int i = 0; i < n; ++i) {
    const ChainStepSpec& s = specs[i];
    const QuantizedLinear& L = *s.layer;
    const StepPlan p = plan_step(L.output_dims(), L.input_dims(), s.rows, grid_);
    cq::ChainStep& st = host_[i];
    std::memset(&st, 0, sizeof(st));
    maps[i] = L.gemv_map(p.rt);
    st.wmap = maps_.as<CUtensorMap>() + i;
    st.scales = L.scales();
    st.biases = L.biases();
    st.bias = L.bias();
    st.x = s.x;
    st.y = s.y;
    st.ldx = s.ldx;
    st.ldy = s.ldy;
    st.M = s.rows;
    st.N = L.output_dims();
    st.K = L.input_dims();
    st.act = s.act;
    st.rt = p.rt;
    st.sb_per_item = p.spi;
    st.kslices = p.kslices;
    st.bands = (st.N + 16 * p.rt - 1) / (16 * p.rt);
    st.mtiles = (s.rows + 15) / 16;
    st.item_base = items_;
    st.items = p.items;
    st.units = st.bands * st.mtiles;
    st.evict_first = st.mtiles == 1 ? 1 : 0;
    for (int d = 0; d < cq::kChainMaxDeps; ++d)
      st.dep[d] = d < static_cast<int>(deps[i].size()) ? deps[i][d] : -1;
    items_ += p.items;
    if (p.kslices > 1) {
      partial_off[i] = partial_floats;
      partial_floats += static_cast<size_t>(st.units) * p.kslices * 16 * p.rt * 16;
      arrive_off[i] = arrive_count;
      arrive_count += st.units;
    }
  }
  check_cuda(cudaMemcpy(maps_.get(), maps.data(), maps.size() * sizeof(CUtensorMap),
                        cudaMemcpyHostToDevice),
             "chain tensor maps");
  partial_ = DeviceBuffer(std::max<size_t>(partial_floats, 1) * sizeof(float));
  arrive_ = DeviceBuffer(std::max<size_t>(arrive_count, 1) * sizeof(unsigned));
  narrive_ = static_cast<int>(arrive_count);
  done_ = DeviceBuffer(static_cast<size_t>(n) * sizeof(unsigned));
  exit_ = DeviceBuffer(sizeof(unsigned));
  abort_ = DeviceBuffer(sizeof(int));
  check_cuda(cudaMemset(arrive_.get(), 0, arrive_.bytes()), "chain counters");
  check_cuda(cudaMemset(done_.get(), 0, done_.bytes()), "chain counters");
  check_cuda(cudaMemset(exit_.get(), 0, exit_.bytes()), "chain counters");
  check_cuda(cudaMemset(abort_.get(), 0, abort_.bytes()), "chain counters");
  for (int i = 0; i < n; ++i) {
    if (host_[i].kslices > 1) {
      host_[i].partial = partial_.as<float>() + partial_off[i];
      host_[i].arrive = arrive_.as<unsigned>() + arrive_off[i];
    }
  }
  // tagged copies of the outputs that later steps read through them
  std::vector<size_t> tagged_off(n, 0);
  std::vector<char> has_tagged(n, 0);
  size_t tagged_words = 0;
  for (int i = 0; i < n; ++i)
    if (tagged_src[i] >= 0) has_tagged[tagged_src[i]] = 1;
  for (int j = 0; j < n; ++j) {
    if (!has_tagged[j]) continue;
    tagged_off[j] = tagged_words;
    tagged_words += static_cast<size_t>(specs[j].rows) * (specs[j].ldy / 2);
  }
  tagged_ = DeviceBuffer(std::max<size_t>(tagged_words, 1) * sizeof(unsigned long long));
  check_cuda(cudaMemset(tagged_.get(), 0, tagged_.bytes()), "chain tagged outputs");
  epoch_ = DeviceBuffer(sizeof(unsigned));
  check_cuda(cudaMemset(epoch_.get(), 0, epoch_.bytes()), "chain epoch");
  for (int j = 0; j < n; ++j) {
    if (!has_tagged[j]) continue;
    host_[j].y_tagged = tagged_.as<unsigned long long>() + tagged_off[j];
    host_[j].y_tagged_ld = specs[j].ldy / 2;
  }
  for (int i = 0; i < n; ++i) {
    if (tagged_src[i] < 0) continue;
    host_[i].x_tagged = host_[tagged_src[i]].y_tagged;
    host_[i].x_tagged_ld = host_[tagged_src[i]].y_tagged_ld;
    host_[i].x_tagged_col = tagged_col[i];
  }
  for (int i = 0; i < n; ++i)
    for (int d : deps[i]) host_[d].signal = 1;
  tagged_src_ = tagged_src;
  tagged_reads_ = 0;
  for (int i = 0; i < n; ++i) tagged_reads_ += tagged_src[i] >= 0 ? 1 : 0;

  steps_ = DeviceBuffer(static_cast<size_t>(n) * sizeof(cq::ChainStep));
  check_cuda(cudaMemcpy(steps_.get(), host_.data(), host_.size() * sizeof(cq::ChainStep),
                        cudaMemcpyHostToDevice),
             "chain steps");
}

void LinearChain::set_profile(bool on) {
  DeviceGuard guard(device_);
  if (!on) {
    trace_ = DeviceBuffer();
    return;
  }
  trace_ = DeviceBuffer(static_cast<size_t>(items_) * cq::kChainTraceStamps * sizeof(uint64_t));
  check_cuda(cudaMemset(trace_.get(), 0, trace_.bytes()), "chain profile");
}

void LinearChain::read_profile(uint64_t* host, size_t len) const {
  const size_t n = static_cast<size_t>(items_) * cq::kChainTraceStamps;
  if (trace_.get() == nullptr) throw_invalid("profiling is not enabled on this chain");
  if (len != n) throw_invalid("the profile holds " + std::to_string(n) + " stamps");
  DeviceGuard guard(device_);
  check_cuda(cudaMemcpy(host, trace_.get(), n * sizeof(uint64_t), cudaMemcpyDeviceToHost),
             "read chain profile");
}

void LinearChain::run(cudaStream_t stream) {
  DeviceContext& ctx = device_context(device_);
  DeviceGuard guard(device_);
  cq::ChainArgs a{};
  a.steps = steps_.as<cq::ChainStep>();
  a.nsteps = static_cast<int>(host_.size());
  a.total_items = items_;
  a.done = done_.as<unsigned>();
  a.arrive = arrive_.as<unsigned>();
  a.narrive = narrive_;
  a.exit_count = exit_.as<unsigned>();
  a.abort_flag = abort_.as<int>();
  a.status = ctx.status;
  a.trace = trace_.as<unsigned long long>();
  a.epoch = epoch_.as<unsigned>();
  check_cuda(cq::launch_chain(dtype_, group_, a, grid_, stream), "linear chain launch");
}

}  // namespace nemotron_cuda
