// The 4-CTA-cluster instance (namespace bcjr::l16c4) of the L=16, k=2, V=1
// kernels in bcjr_l16.cu: two sequences in flight per cluster in the backward
// as well, on the 132 SMs that clusters of 4 tile.  The dispatcher in
// bcjr_l16.cu runs it beside the 2-CTA instance.
#define BCJR_L16_CL 4
#include "bcjr_l16.cu"
