"""B200-native token sampler for the QEdge decode loop.

Drop-in for QEdge's ``BatchSampler`` (``src/compute/sampler.py:22-41``):
logits ``[B, V]`` in, token ids ``[B]`` out, computed by hand-written sm_100a
CUDA kernels behind the C ABI declared in ``include/qedge_sample.h``.
"""
__all__ = ["QESampler", "SamplingParams", "SamplingBatch"]


def __getattr__(name):
    if name == "QESampler":
        from .sampler import QESampler
        return QESampler
    if name == "SamplingParams":
        from .sampling_params import SamplingParams
        return SamplingParams
    if name == "SamplingBatch":
        from .batch import SamplingBatch
        return SamplingBatch
    raise AttributeError(name)
