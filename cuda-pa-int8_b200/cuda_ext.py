"""Module-name shim: with this directory first on sys.path, `from cuda_ext import VARIANTS`
(the import the reference's tests and benches use) resolves to pa_b200.cuda_ext."""

from pa_b200.cuda_ext import (  # noqa: F401
    VARIANTS,
    VARIANTS_INT8,
    paged_decode_attention,
    quantize_into_cache,
)
