"""Model-family registry (API of kvcompress/adapters/registry.py).

Maps Hugging Face ``config.model_type`` to a module exposing
``install(model, cache_manager)``.  Every family the reference lists uses the
standard cache layout, which the ``DynamicCache`` subclass of
``HuggingFaceAdapter`` covers, so they all resolve to the generic no-op shim
(``kvcompress_b200.adapters.families``); the registry is where a family with
its own cache layout would hook in.  Register custom families before an
adapter is constructed (the table is not locked).
"""

from __future__ import annotations

import importlib
import logging
from typing import Any, Callable

log = logging.getLogger(__name__)

_GENERIC = "kvcompress_b200.adapters.families"

REGISTRY: dict[str, str] = {t: _GENERIC for t in (
    "llama", "mistral", "qwen2", "qwen2_moe", "gemma", "gemma2", "phi", "phi3", "mixtral", "falcon",
    "deepseek", "internlm")}


def known_model_types() -> list[str]:
    """Every registered ``model_type``, sorted."""
    return sorted(REGISTRY)


def resolve(model_type: str) -> str | None:
    """Dotted path of the module handling ``model_type``, or None."""
    return REGISTRY.get(model_type)


def register(model_type: str, module_path: str) -> None:
    """Add a family shim; ``ValueError`` if ``model_type`` is taken."""
    if model_type in REGISTRY:
        raise ValueError(f"model_type {model_type!r} already registered")
    REGISTRY[model_type] = module_path


def install(model: Any, cache_manager: Any, model_type: str) -> Callable[[], None] | None:
    """Run the family shim's ``install``; unknown types take the generic path
    (a warning, then ``None``)."""
    path = resolve(model_type)
    if path is None:
        log.warning("kvcompress: no shim for model_type=%s; using generic interception", model_type)
        from kvcompress_b200.adapters.huggingface import generic_install

        generic_install(model, cache_manager)
        return None
    return importlib.import_module(path).install(model, cache_manager)
