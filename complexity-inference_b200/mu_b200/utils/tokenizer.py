"""Optional tokenizer loading (text I/O is outside the forward step).

The reference wraps a HuggingFace AutoTokenizer (mu_inference/utils/
tokenizer.py:17-191).  Here a tokenizer is loaded only when the model
directory ships one and ``transformers`` can read it offline; otherwise the
engines take token ids directly.
"""

from __future__ import annotations

from pathlib import Path
from typing import Optional


def load_tokenizer(model_path: str) -> Optional[object]:
    p = Path(model_path)
    if not any((p / f).exists() for f in ("tokenizer.json", "tokenizer.model",
                                          "tokenizer_config.json")):
        return None
    try:
        from transformers import AutoTokenizer

        return AutoTokenizer.from_pretrained(str(p), local_files_only=True)
    except Exception:
        return None
