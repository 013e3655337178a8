// mmvq_q6k_c8.cu -- instantiations of the Q6_K MMVQ kernel template for 8
// activation column(s); split per batch width so the build compiles them in
// parallel.
#include "mmvq_q6k_impl.cuh"

namespace abra {
const Q6Table &q6_table_c8() {
    static const Q6Table t = make_q6_table<8>();
    return t;
}
}  // namespace abra

ABRA_ERROR_WORD_ACCESSOR(error_word_mmvq_q6k_c8)
