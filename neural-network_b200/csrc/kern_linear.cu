// Instantiations of linear_kernel (forward.cuh): 4 type pairs x 5 epilogues x
// input LayerNorm on/off x 2 column widths, exposed as a pointer table.
#include "forward.cuh"
#include "kern_table.cuh"

namespace specdec {

namespace {
template <typename W, typename A, int EPI, bool LN>
const void *pick_nc(int nc) {
  return nc == 4 ? reinterpret_cast<const void *>(linear_kernel<W, A, EPI, LN, 4>)
                 : reinterpret_cast<const void *>(linear_kernel<W, A, EPI, LN, 2>);
}
template <typename W, typename A, int EPI>
const void *pick_ln(int ln, int nc) {
  return ln ? pick_nc<W, A, EPI, true>(nc) : pick_nc<W, A, EPI, false>(nc);
}
template <typename W, typename A>
const void *pick_epi(int epi, int ln, int nc) {
  switch (epi) {
    case kEpiStore: return pick_ln<W, A, kEpiStore>(ln, nc);
    case kEpiResid: return pick_ln<W, A, kEpiResid>(ln, nc);
    case kEpiQKV: return pick_ln<W, A, kEpiQKV>(ln, nc);
    case kEpiSwiGLU: return pick_ln<W, A, kEpiSwiGLU>(ln, nc);
    case kEpiGelu: return pick_ln<W, A, kEpiGelu>(ln, nc);
    default: return nullptr;
  }
}
}  // namespace

const void *linear_kernel_fn(int w8, int abf, int epi, int ln, int nc) {
  if (w8 && abf) return pick_epi<int8_t, __nv_bfloat16>(epi, ln, nc);
  if (w8) return pick_epi<int8_t, float>(epi, ln, nc);
  if (abf) return pick_epi<float, __nv_bfloat16>(epi, ln, nc);
  return pick_epi<float, float>(epi, ln, nc);
}

}  // namespace specdec
