// Host runtime for the paged KV cache: a block allocator with reference
// counts (prefix sharing) and the prefill metadata builder.
//
// Exposed as torch.classes._b200_C.BlockAllocator and
// torch.ops._b200_C.build_prefill_meta (CPU tensors). These are the hot host
// paths of the scheduler: at 256-request batches the per-token slot mapping
// of a 16K-token prefill chunk is built here in one pass instead of in Python.
//
// Reference parity: the reference relies on upstream vLLM's KV-cache manager
// (Python); this runtime owns its scheduler, so the block manager is native.
#include <torch/custom_class.h>
#include <torch/library.h>
#include <torch/torch.h>

#include <algorithm>
#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>

namespace b200 {

struct BlockAllocator : torch::CustomClassHolder {
  std::vector<int32_t> free_list;  // LIFO
  std::vector<int32_t> refcnt;
  int64_t reserved;

  BlockAllocator(int64_t num_blocks, int64_t reserved_blocks) : reserved(reserved_blocks) {
    TORCH_CHECK(num_blocks > reserved_blocks && reserved_blocks >= 0, "bad block counts");
    refcnt.assign(num_blocks, 0);
    free_list.reserve(num_blocks);
    // Hand out low block ids first (pop from the back).
    for (int64_t b = num_blocks - 1; b >= reserved_blocks; --b) free_list.push_back((int32_t)b);
  }

  int64_t num_free() const { return (int64_t)free_list.size(); }
  int64_t num_total() const { return (int64_t)refcnt.size(); }

  at::Tensor allocate(int64_t n) {
    TORCH_CHECK(n >= 0, "allocate: negative count");
    if ((int64_t)free_list.size() < n)
      throw std::runtime_error("BlockAllocator: out of KV blocks (need " + std::to_string(n) +
                               ", free " + std::to_string(free_list.size()) + ")");
    auto out = at::empty({n}, at::TensorOptions().dtype(at::kInt));
    int32_t* p = out.data_ptr<int32_t>();
    for (int64_t i = 0; i < n; ++i) {
      const int32_t b = free_list.back();
      free_list.pop_back();
      refcnt[b] = 1;
      p[i] = b;
    }
    return out;
  }

  void incref(const at::Tensor& blocks) {
    auto b = blocks.to(at::kInt).contiguous();
    const int32_t* p = b.data_ptr<int32_t>();
    for (int64_t i = 0; i < b.numel(); ++i) {
      TORCH_CHECK(p[i] >= reserved && p[i] < (int32_t)refcnt.size() && refcnt[p[i]] > 0,
                  "incref: block not allocated");
      ++refcnt[p[i]];
    }
  }

  void free(const at::Tensor& blocks) {
    auto b = blocks.to(at::kInt).contiguous();
    const int32_t* p = b.data_ptr<int32_t>();
    for (int64_t i = 0; i < b.numel(); ++i) {
      const int32_t id = p[i];
      TORCH_CHECK(id >= reserved && id < (int32_t)refcnt.size(), "free: bad block id");
      TORCH_CHECK(refcnt[id] > 0, "free: double free of block ", id);
      if (--refcnt[id] == 0) free_list.push_back(id);
    }
  }

  int64_t block_refcount(int64_t id) const { return refcnt.at(id); }
};

// For a prefill batch of S sequence pieces: piece s covers positions
// [ctx_start[s], ctx_start[s] + q_len[s]) of its sequence, whose block row
// is block_table[s]. Returns (positions int64 [T], slots int64 [T]).
std::tuple<at::Tensor, at::Tensor> build_prefill_meta(const at::Tensor& block_table,
                                                      const at::Tensor& ctx_start,
                                                      const at::Tensor& q_len,
                                                      int64_t block_size) {
  TORCH_CHECK(!block_table.is_cuda() && block_table.scalar_type() == at::kInt, "cpu int32 table");
  auto bt = block_table.contiguous();
  auto cs = ctx_start.to(at::kInt).contiguous();
  auto ql = q_len.to(at::kInt).contiguous();
  const int64_t S = ql.numel();
  const int64_t maxb = bt.size(1);
  int64_t T = 0;
  for (int64_t s = 0; s < S; ++s) T += ql.data_ptr<int32_t>()[s];
  auto pos = at::empty({T}, at::TensorOptions().dtype(at::kLong));
  auto slots = at::empty({T}, at::TensorOptions().dtype(at::kLong));
  int64_t* pp = pos.data_ptr<int64_t>();
  int64_t* sp = slots.data_ptr<int64_t>();
  const int32_t* btp = bt.data_ptr<int32_t>();
  int64_t t = 0;
  for (int64_t s = 0; s < S; ++s) {
    const int64_t c0 = cs.data_ptr<int32_t>()[s];
    const int64_t n = ql.data_ptr<int32_t>()[s];
    for (int64_t j = 0; j < n; ++j, ++t) {
      const int64_t p = c0 + j;
      const int64_t bi = p / block_size;
      TORCH_CHECK(bi < maxb, "build_prefill_meta: position beyond the block table");
      pp[t] = p;
      sp[t] = (int64_t)btp[s * maxb + bi] * block_size + p % block_size;
    }
  }
  return {pos, slots};
}

}  // namespace b200

TORCH_LIBRARY_FRAGMENT(_b200_C, m) {
  m.class_<b200::BlockAllocator>("BlockAllocator")
      .def(torch::init<int64_t, int64_t>())
      .def("num_free", &b200::BlockAllocator::num_free)
      .def("num_total", &b200::BlockAllocator::num_total)
      .def("allocate", &b200::BlockAllocator::allocate)
      .def("incref", &b200::BlockAllocator::incref)
      .def("free", &b200::BlockAllocator::free)
      .def("block_refcount", &b200::BlockAllocator::block_refcount);
  m.def("build_prefill_meta(Tensor block_table, Tensor ctx_start, Tensor q_len, int block_size) -> (Tensor, Tensor)",
        &b200::build_prefill_meta);
}
