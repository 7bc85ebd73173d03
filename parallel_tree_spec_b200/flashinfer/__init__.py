"""The reference's ``parallel_tree_spec.flashinfer`` subpackage, module for module.

``cache_manager`` and ``attention_wrapper`` are the package's own modules
under the reference's import paths; ``attention``, ``modeling_llama`` and
``monkey_patch`` patch a Hugging Face Llama model so that its attention runs
through ``BeFlashinferWrapper`` (``flashinfer/__init__.py``,
``flashinfer/monkey_patch.py:95-123``).  Nothing here imports the FlashInfer
library.
"""
from .cache_manager import KvCacheBatchPosition, KvCachePool, RequestKvCache, getKvCacheBatchPosition
from .attention_wrapper import BeFlashinferWrapper
from .monkey_patch import apply_flashinfer_kernel_to_llama
