"""Family shim for the standard cache layout (the reference's llama.py,
mistral.py, qwen.py, gemma.py, phi.py, mixtral.py, falcon.py, deepseek.py,
internlm.py are all this no-op): the ``DynamicCache`` subclass installed by
``HuggingFaceAdapter`` already sees every cache write and read."""

from __future__ import annotations

from typing import Any


def install(model: Any, cache_manager: Any) -> None:
    """Nothing to hook for the standard layout."""
    return None
