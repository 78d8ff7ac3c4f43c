"""B200-native (sm_100a) decode-time KV eviction: fused decode attention + H2O
scores, ragged per-head selection and compaction behind a C ABI
(include/ce_api.h), with a Python mirror of the reference overlay's hooks.

Submodules: capi (ctypes binding), kernels (torch front end), runtime (the
gstar_evict hook API), policy (policy vocabulary and validation), engine
(ragged continuous-batch driver), tp (KV-head sharding over NCCL).
"""
__version__ = "0.1.0"
