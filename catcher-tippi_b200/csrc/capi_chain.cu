// extern "C" boundary of the persistent linear-chain executor (include/cqchain.h).
#include <memory>
#include <vector>

#include "capi_guard.hpp"
#include "cqchain.h"
#include "linear_chain.hpp"

struct cq_linear_chain {
  std::unique_ptr<nemotron_cuda::LinearChain> impl;
};

namespace {
using nemotron_cuda::guarded;
using nemotron_cuda::need_handle;
}  // namespace

extern "C" {

cq_status cq_linear_chain_create(const cq_chain_step* steps, int32_t count, cq_linear_chain** out) {
  return guarded([&] {
    need_handle(out, "out");
    *out = nullptr;
    need_handle(steps, "steps");
    if (count <= 0) nemotron_cuda::throw_invalid("a linear chain needs at least one step");
    std::vector<nemotron_cuda::ChainStepSpec> specs(count);
    for (int32_t i = 0; i < count; ++i) {
      need_handle(steps[i].layer, "layer");
      specs[i] = nemotron_cuda::ChainStepSpec{steps[i].layer->impl, steps[i].x, steps[i].ldx,
                                              steps[i].rows, steps[i].y, steps[i].ldy, steps[i].act};
    }
    auto h = std::make_unique<cq_linear_chain>();
    h->impl = std::make_unique<nemotron_cuda::LinearChain>(specs);
    *out = h.release();
  });
}

cq_status cq_linear_chain_run(cq_linear_chain* chain, void* stream) {
  return guarded([&] {
    need_handle(chain, "chain");
    chain->impl->run(static_cast<cudaStream_t>(stream));
  });
}

cq_status cq_linear_chain_step_info(const cq_linear_chain* chain, int32_t index,
                                    int32_t* rows_per_item, int32_t* subblocks_per_item,
                                    int32_t* kslices, int32_t* first_item, int32_t* items,
                                    int32_t* reads_tagged, int32_t* waits_for) {
  return guarded([&] {
    need_handle(chain, "chain");
    if (index < 0 || index >= chain->impl->steps())
      nemotron_cuda::throw_invalid("step index out of range");
    const cq::ChainStep& st = chain->impl->step_plan(index);
    if (rows_per_item) *rows_per_item = 16 * st.rt;
    if (subblocks_per_item) *subblocks_per_item = st.sb_per_item;
    if (kslices) *kslices = st.kslices;
    if (first_item) *first_item = st.item_base;
    if (items) *items = st.items;
    if (reads_tagged) *reads_tagged = chain->impl->tagged_source(index);
    if (waits_for)
      for (int d = 0; d < cq::kChainMaxDeps; ++d) waits_for[d] = st.dep[d];
  });
}

cq_status cq_linear_chain_profile(cq_linear_chain* chain, int32_t enable) {
  return guarded([&] {
    need_handle(chain, "chain");
    chain->impl->set_profile(enable != 0);
  });
}

cq_status cq_linear_chain_read_profile(const cq_linear_chain* chain, uint64_t* stamps, size_t len) {
  return guarded([&] {
    need_handle(chain, "chain");
    need_handle(stamps, "stamps");
    chain->impl->read_profile(stamps, len);
  });
}

int32_t cq_linear_chain_items(const cq_linear_chain* chain) {
  return chain == nullptr ? 0 : chain->impl->items();
}

int32_t cq_linear_chain_grid(const cq_linear_chain* chain) {
  return chain == nullptr ? 0 : chain->impl->grid();
}

void cq_linear_chain_destroy(cq_linear_chain* chain) { delete chain; }

}  // extern "C"
