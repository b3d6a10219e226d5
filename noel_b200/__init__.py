"""B200 token-sampling path with the reference sampler's semantics
(Sain-Kai/noel src/sampler.c), as hand-written sm_100a CUDA kernels behind
the reference C ABI (include/sampler.h) plus batched device entry points
(include/noel_sampler_cuda.h)."""
