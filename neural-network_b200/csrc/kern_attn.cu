// Instantiations of attention_kernel (forward.cuh): query type x cache type x
// head dimension x queries per CTA, exposed as a pointer table.
#include "forward.cuh"
#include "kern_table.cuh"

namespace specdec {

namespace {
template <typename AT, typename KT, int D>
const void *pick_qt(int qt) {
  switch (qt) {
    case 1: return reinterpret_cast<const void *>(attention_kernel<AT, KT, D, 1>);
    case 2: return reinterpret_cast<const void *>(attention_kernel<AT, KT, D, 2>);
    case 4: return reinterpret_cast<const void *>(attention_kernel<AT, KT, D, 4>);
    case 8: return reinterpret_cast<const void *>(attention_kernel<AT, KT, D, 8>);
    default: return nullptr;
  }
}
template <typename AT, typename KT>
const void *pick_d(int D, int qt) {
  switch (D) {
    case 4: return pick_qt<AT, KT, 4>(qt);
    case 8: return pick_qt<AT, KT, 8>(qt);
    case 16: return pick_qt<AT, KT, 16>(qt);
    case 32: return pick_qt<AT, KT, 32>(qt);
    case 64: return pick_qt<AT, KT, 64>(qt);
    case 128: return pick_qt<AT, KT, 128>(qt);
    default: return nullptr;
  }
}
template <typename AT>
const void *pick_kt(int kt, int D, int qt) {
  switch (kt) {
    case 0: return pick_d<AT, float>(D, qt);
    case 1: return pick_d<AT, __nv_bfloat16>(D, qt);
    case 2: return pick_d<AT, int8_t>(D, qt);
    default: return nullptr;
  }
}
}  // namespace

const void *attention_kernel_fn(int abf, int kt, int D, int qt) {
  return abf ? pick_kt<__nv_bfloat16>(kt, D, qt) : pick_kt<float>(kt, D, qt);
}

}  // namespace specdec
