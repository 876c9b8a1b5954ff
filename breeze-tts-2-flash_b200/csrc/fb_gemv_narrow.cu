// flashb: the tensor-core GEMV built for 32 KB stages (16 rows x 1024 columns): used when activation rows leave too
// little shared memory for a deep ring of 64 KB stages (e.g. 16 rows of the 2048-wide projections, eight streams
// served together: two 64 KB stages, but four 32 KB ones).
#define FB_ST_KC 1024
#include "fb_gemv_core.cuh"

namespace fb {

int gemv_mma_narrow(GemvArgs& a, int epi, bool norm, cudaStream_t st, int xchunk, int min_nst) {
  if (epi == 0 && norm) return launch_mma_t<0, true>(a, st, xchunk, min_nst);
  if (epi == 0) return launch_mma_t<0, false>(a, st, xchunk, min_nst);
  if (epi == 1) return launch_mma_t<1, false>(a, st, xchunk, min_nst);
  if (epi == 2 && norm) return launch_mma_t<2, true>(a, st, xchunk, min_nst);
  if (epi == 2) return launch_mma_t<2, false>(a, st, xchunk, min_nst);
  fbh::set_msg("gemv: no 32 KB-stage build for epilogue %d", epi);
  return FB_ERR_UNSUPPORTED;
}

}  // namespace fb
