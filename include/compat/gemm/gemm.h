/* gemm/gemm.h -- the path the reference's sources include its GEMM interface
 * by (reference src/model.h:46, tests/test_gemm_naive.c:16); it resolves to
 * this engine's include/gemm.h, so a reference caller compiled with
 * -I include -I include/compat sees the engine's declarations. */
#include "../../gemm.h"
