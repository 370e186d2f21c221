"""B200 (sm_100a) attention step of picolm_qwen behind a C ABI (include/picoattn.h).

The product is ``libpicoattn.so`` (hand-written CUDA, built in tree by
``picolm_qwen_b200.build``).  This package holds the ctypes binding
(``picolm_qwen_b200.abi``) that tests and the benchmark use to call it; there is
no fallback path: if the shared library is missing, importing the binding
raises.
"""
from .abi import (  # noqa: F401
    PICOATTN_OK, PICOATTN_EINVAL, PICOATTN_EUNSUPPORTED, PICOATTN_ERANGE, PICOATTN_ENOSPACE,
    PICOATTN_ECUDA, PICOATTN_EDEVICE, ROPE_NEOX, ROPE_INTERLEAVED, Config, lib, check,
)
