// mmvq_c6.cu -- instantiations of the MMVQ kernel template for 6 activation
// column(s); split per batch width so the build compiles them in parallel.
#include "mmvq_impl.cuh"

namespace abra {
const MmvqTable &mmvq_table_c6() {
    static const MmvqTable t = make_mmvq_table<6>();
    return t;
}
}  // namespace abra

ABRA_ERROR_WORD_ACCESSOR(error_word_mmvq_c6)
