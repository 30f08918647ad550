"""B200-native (sm_100a) sparse submanifold convolution path of mosure/bevy_synth's
TRELLIS.2 sparse decoders: coordinate hash + neighbor map, tcgen05 gather-GEMM
conv with fused bias/residual/LayerNorm/SiLU epilogues, channel-to-space
upsample, behind the C ABI of include/sparseconv.h (libsparseconv.so).

``flex_gmm`` mirrors the reference operator API (crate burn_flex_gmm);
``blocks`` holds the decoder blocks; ``sharding`` the multi-GPU partitioning;
``synth`` the seeded synthetic workloads.
"""
from ._lib import SparseConvError  # noqa: F401

__all__ = ["SparseConvError"]
