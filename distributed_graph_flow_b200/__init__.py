"""B200-native (sm_100a) sampler and sparse aggregation for Distributed Graph Flow.

Drop-in for DGF's in-memory k-hop temporal neighbour sampler
(``dgf.sampling.create_sampler`` / ``Sampler.sample``) and for the sparse
neighbour aggregation of its GNN layers (segment_sum / SpMM), with the
compute in hand-written CUDA kernels behind the C ABI in include/dgfx.h.
"""

__version__ = "0.1.0"
