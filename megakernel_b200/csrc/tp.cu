// Tensor-parallel instantiations of the decode megakernel, and the TP = 1
// instances with the two-level attention merge (long context).
//
// configs[4](b): the MLP (gate/up rows, down columns) and the LM head (vocab
// rows) are split over TP GPUs; attention and the O projection stay
// replicated.  Per layer each rank writes its partial down projection into
// every rank's X hop over NVLink (system-scope tagged words through CUDA IPC
// mappings) and every rank sums the TP partials in rank order; per token each
// CTA's (max, index) pair goes to every rank.  The reference is single-GPU and
// has no counterpart.  Kept in its own translation unit so that it compiles in
// parallel with megakernel.cu; the host side (state, IPC, C ABI) lives there.
#include "decode_kernel.cuh"

namespace mk_tp {

template <class S, int TP, bool M2>
const void* entry(size_t* hop_words) {
  *hop_words = (size_t)mk::HopLayout<S, TP>::TOTAL;
  return reinterpret_cast<const void*>(&mk::decode_kernel<S, TP, M2>);
}

// Kernel of (shape id, TP size, two-level merge) and its hop-buffer size in
// 64-bit words, or nullptr if that combination is not compiled.  TP kernels
// always carry the two-level merge.
const void* kernel(int shape_id, int tp, bool m2, size_t* hop_words) {
  if (tp == 1) {
    if (!m2) return nullptr;   // the direct-merge TP = 1 kernels live in megakernel.cu
    if (shape_id == 0) return entry<mk::ShapeD64, 1, true>(hop_words);
    if (shape_id == 1) return entry<mk::ShapeD128, 1, true>(hop_words);
    if (shape_id == 2) return entry<mk::ShapeTiny, 1, true>(hop_words);
    return nullptr;
  }
  if (!m2) return nullptr;
  if (shape_id == 0) {
    if (tp == 2) return entry<mk::ShapeD64, 2, true>(hop_words);
    if (tp == 4) return entry<mk::ShapeD64, 4, true>(hop_words);
    if (tp == 8) return entry<mk::ShapeD64, 8, true>(hop_words);
  } else if (shape_id == 2) {
    if (tp == 2) return entry<mk::ShapeTiny, 2, true>(hop_words);
  }
  return nullptr;
}

}  // namespace mk_tp
