"""Placeholder of the reference's CPU CompressAI-RANS backend.

The reference wraps ``compressai.ans.RansEncoder/RansDecoder``
(coders/compressai_ans.py:14-88).  That CPU coder is outside the B200 hot
path this package rebuilds; the constructor keeps the reference's
dependency behaviour (``CoderDependencyError`` when CompressAI is missing)
so ``create_coder("compressai-rans")`` fails the same way.
"""

from __future__ import annotations

from .errors import CoderDependencyError


class CompressAIANSBackend:
    name = "compressai-rans"
    schema_version = 1

    def __init__(self) -> None:
        try:
            from compressai import ans  # noqa: F401
        except (ImportError, ModuleNotFoundError) as exc:
            raise CoderDependencyError(
                "CompressAI RANS is unavailable; install fast-compressai[compressai]"
            ) from exc
        raise CoderDependencyError(
            "the CPU CompressAI-RANS session backend is not part of fast_compressai's B200 build; "
            "use compressai.ans directly"
        )
