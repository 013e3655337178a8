// mmvq_c5.cu -- instantiations of the MMVQ kernel template for 5 activation
// column(s); split per batch width so the build compiles them in parallel.
#include "mmvq_impl.cuh"

namespace abra {
const MmvqTable &mmvq_table_c5() {
    static const MmvqTable t = make_mmvq_table<5>();
    return t;
}
}  // namespace abra

ABRA_ERROR_WORD_ACCESSOR(error_word_mmvq_c5)
