"""kvengine_b200: kvengine's greedy speculative-decoding path on B200 (sm_100a).

Keeps the reference's names for the spec path (kvengine/__init__.py:1-52):
`speculative_greedy`, `SpecDecodeResult`, `forward_with_own_cache`,
`PagedKVCache`, `PagedSequenceCache`, `BlockManager`, `OutOfBlocks`,
`DoubleFree`, `greedy_paged`, `AUTO_EOS`, `DEFAULT_BLOCK_SIZE`; adds
`speculative_greedy_batch`, `greedy_batch` and `Model`.

The compute runs in `libkvengine_b200.so` (C ABI in include/kvengine_b200.h);
importing this package does not load it, the first op does, and fails loudly
if it is missing.
"""

from .blocks import BlockManager, DoubleFree, OutOfBlocks
from .config import PRESETS, QWEN2_0_5B, QWEN2_3B, TINY, ModelConfig
from .decode import AUTO_EOS, GenerationResult, greedy_batch, greedy_paged
from .forward import forward_with_own_cache
from .model import Model, as_model
from .paged import DEFAULT_BLOCK_SIZE, PagedKVCache, PagedSequenceCache
from .serving import SpecServer
from .speculative import SpecDecodeResult, SpecEngine, speculative_greedy, speculative_greedy_batch

__all__ = [
    "AUTO_EOS", "DEFAULT_BLOCK_SIZE", "BlockManager", "DoubleFree", "GenerationResult", "Model",
    "ModelConfig", "OutOfBlocks", "PRESETS", "PagedKVCache", "PagedSequenceCache", "QWEN2_0_5B", "QWEN2_3B",
    "SpecDecodeResult", "SpecEngine", "TINY", "as_model", "forward_with_own_cache", "greedy_batch",
    "greedy_paged", "speculative_greedy", "speculative_greedy_batch", "SpecServer",
]
