"""K8/V4 cache formats: page geometry, quantization oracles, byte pack, views."""
from .layout import (  # noqa: F401
    B200_FORMAT, CACHE_DTYPE, FORMATS, REF_FORMAT, KVFormat, PageLayout, b200_layout, ref_layout,
)
