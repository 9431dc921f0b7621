"""nano_vllm_b200 -- B200 (sm_100a) attention hot path of nano-vllm-metal.

Drop-in for the reference's ``layers/attention`` operators and ``cache/paged``
page pools: ``paged_attention``, ``flash_attention``, ``TinyKvPagedPool``,
``TinyKvPagedCache``, ``BatchingKvCache`` keep the reference's names and
signatures (the reference's ``PrefixCache`` runs unchanged over these pools); the
kernels live in ``libnvm_attn.so`` (C ABI in ``include/nvm_attn.h``).
"""

from .layers.attention import (  # noqa: F401
    causal_mask,
    flash_attention,
    paged_attention,
    scaled_dot_product_attention_grouped,
)
from .cache.kv_cache import BatchingKvCache, TinyKvCache  # noqa: F401
from .cache.paged import (  # noqa: F401
    DevicePageTable,
    PagedKvMetadata,
    TinyKvPagedCache,
    TinyKvPagedPool,
    write_slots,
)
from .spec_verify import VerifyResult, verify_accept  # noqa: F401
from . import _native  # noqa: F401

__version__ = "0.1.0"
