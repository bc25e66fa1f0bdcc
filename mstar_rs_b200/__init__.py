"""B200-native batched token sampler for the mstar-rs decode hot path.

The sampling arithmetic runs in hand-written sm_100a CUDA
(mstar_rs_b200/csrc/sampler.cu) behind a C ABI (include/mstar_sampler.h);
`sampling` mirrors the Python sampler interface the reference's engines call
(SamplingConfig / Sampler / SamplerBuffers / SeenTokenMask /
CudaGraphableSampler).
"""
__version__ = "0.1.0"
