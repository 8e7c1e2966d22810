// b2_tc.cu -- tensor-core bank product (tcgen05 kind::i8). Not yet enabled: every bank reports not-ready, so the
// engine uses the CUDA-core product.
#include "b2_tc.cuh"

namespace b2 {

int tc_min_rows_default() { return 1 << 30; }
int tc_bank_build(TcBank& t, const int16_t*, int nin, int nout) {
    t.ready = 0;
    t.nin = nin;
    t.nout = nout;
    return 1;
}
void tc_bank_free(TcBank& t) { t.ready = 0; }
int tc_rows_alloc(TcRows&, int, int) { return 0; }
void tc_rows_free(TcRows&) {}
void tc_planes(TcRows&, const int32_t*, int, int, cudaStream_t) {}
int tc_bank(const TcBank&, TcRows&, int, int, const int32_t*, const int64_t*, const int32_t*, const int64_t*, int64_t*,
            int, const int32_t*, const int32_t*, const int32_t*, cudaStream_t) {
    return (int)cudaErrorNotSupported;
}

}  // namespace b2
