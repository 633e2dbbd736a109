"""pse -- B200-native (sm_100a) speculative draft -> verify -> accept/reject ->
commit engine over a device-resident paged KV cache.

Drop-in for vedantjain09/paged-speculative-engine's hot path: the module and
function names mirror engine/paged_cache.py, engine/batched_forward.py,
engine/speculative.py, engine/scheduler.py and engine/generate.py.  All
compute runs in libpse.so (hand-written CUDA kernels behind a C ABI,
include/pse.h) on torch's current stream; there is no CPU path.
"""
from .batched_forward import batched_forward_append
from .generate import speculative_generate_batched
from .model import LlamaConfig, ModelConfig, TinyGPT, TinyLlama
from .paged_cache import BlockAllocator, PagedKVCache
from .scheduler import Request, RequestResult, run_continuous_speculative_batches
from .plain import run_plain_continuous_batches
from .speculative import BatchStepResult, batched_speculative_step, prefill_request, prefill_requests
from .tree import batched_tree_speculative_step, speculative_generate_tree

__all__ = [
    "BatchStepResult", "BlockAllocator", "LlamaConfig", "ModelConfig", "PagedKVCache", "Request",
    "RequestResult", "TinyGPT", "TinyLlama", "batched_forward_append", "batched_speculative_step",
    "batched_tree_speculative_step", "speculative_generate_tree",
    "prefill_request", "prefill_requests", "run_continuous_speculative_batches", "run_plain_continuous_batches",
    "speculative_generate_batched",
]
