"""JSON parsing with the process-wide size and nesting caps.

Reference: nano-vllm-java/src/main/java/com/igormaznitsa/nanollvm/internal/Json.java (a minimal parser that
rejects documents deeper than the depth cap or longer than the character cap; caps from ResourceLimits).
Here the standard library parses; a linear pre-scan enforces the caps before it does, so a hostile
config.json / tokenizer.json cannot exhaust the interpreter's recursion or memory.
"""
from __future__ import annotations

import json
from typing import Any, Optional, Union

from ..exceptions import ModelLoadException
from .limits import ResourceLimits


def max_depth(text: str) -> int:
    depth = best = 0
    in_str = esc = False
    for ch in text:
        if in_str:
            if esc:
                esc = False
            elif ch == "\\":
                esc = True
            elif ch == '"':
                in_str = False
        elif ch == '"':
            in_str = True
        elif ch in "[{":
            depth += 1
            best = max(best, depth)
        elif ch in "]}":
            depth -= 1
    return best


def loads(data: Union[str, bytes], what: str = "JSON", depth_cap: Optional[int] = None,
          size_cap: Optional[int] = None) -> Any:
    depth_cap = ResourceLimits.JSON_MAX_DEPTH if depth_cap is None else depth_cap
    size_cap = ResourceLimits.JSON_MAX_BYTES if size_cap is None else size_cap
    if len(data) > size_cap:
        raise ModelLoadException(f"{what}: {len(data)} bytes exceeds the JSON size cap ({size_cap})")
    text = data.decode("utf-8") if isinstance(data, (bytes, bytearray)) else data
    d = max_depth(text)
    if d > depth_cap:
        raise ModelLoadException(f"{what}: nesting depth {d} exceeds the JSON depth cap ({depth_cap})")
    try:
        return json.loads(text)
    except json.JSONDecodeError as e:
        raise ModelLoadException(f"{what}: malformed JSON: {e}") from e


def load_file(path: str, what: Optional[str] = None) -> Any:
    import os
    size = os.path.getsize(path)
    if size > ResourceLimits.JSON_MAX_BYTES:
        raise ModelLoadException(f"{path}: {size} bytes exceeds the JSON size cap ({ResourceLimits.JSON_MAX_BYTES})")
    with open(path, "rb") as f:
        return loads(f.read(), what or path)
