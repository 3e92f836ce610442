"""B200-native (sm_100a) attention hot path of Nanosaur2: the DiT's joint image+text attention with its
q/k RMSNorm + 2D RoPE prologue, and the Gemma3-270M causal GQA attention, behind a C ABI
(include/nsattn.h, libnsattn.so) with a Python mirror of the reference's ``ops.attention`` /
``ops.headNorm`` operator surface."""

from ._lib import NsaError, version  # noqa: F401

__all__ = ["NsaError", "version", "ops", "blocks", "sharding"]
