// mmvq_c7.cu -- instantiations of the MMVQ kernel template for 7 activation
// column(s); split per batch width so the build compiles them in parallel.
#include "mmvq_impl.cuh"

namespace abra {
const MmvqTable &mmvq_table_c7() {
    static const MmvqTable t = make_mmvq_table<7>();
    return t;
}
}  // namespace abra

ABRA_ERROR_WORD_ACCESSOR(error_word_mmvq_c7)
