"""Context limits and KV-cache sizing; a mirror of the reference's
src/core/context.ts (ahpah-dev/WebGPU 0.9.0), same rules and messages."""
from __future__ import annotations

MAX_CONTEXT = 32768
MAX_MESSAGE_CHARS = 1048576


def _is_int(v) -> bool:
    return isinstance(v, int) and not isinstance(v, bool) or (isinstance(v, float) and v == v and v == int(v))


def validate_context(context, model_limit: int = MAX_CONTEXT) -> None:
    """context.ts:5-8."""
    if not _is_int(context) or context < 256 or context > MAX_CONTEXT:
        raise ValueError(f"Context must be an integer from 256 to {MAX_CONTEXT} tokens.")
    if context > model_limit:
        raise ValueError(f"This model declares a {model_limit:,}-token context. Choose a smaller context.")


def output_limit(requested, prompt_tokens: int, context: int) -> int:
    """context.ts:9-13."""
    if not _is_int(requested) or requested < 1 or requested > MAX_CONTEXT:
        raise ValueError(f"maxTokens must be 1–{MAX_CONTEXT}.")
    if prompt_tokens >= context:
        raise ValueError(f"The prompt has {prompt_tokens:,} tokens; the context limit is {context:,}. "
                         "Start a new chat or reload with a longer context.")
    return int(min(requested, context - prompt_tokens))


def attention_memory(c, context: int, batch: int) -> dict:
    """context.ts:16-24 — per-layer KV ring capacities and fp32 K+V bytes. Sliding
    layers keep the window plus the rest of a prompt batch."""
    caps = []
    for l in range(c.layers):
        if c.family == "gemma3":
            caps.append(min(context, c.window + batch - 1) if l % c.period != c.period - 1 else context)
        elif getattr(c, "sliding_window", 0) > 0:
            caps.append(min(context, c.sliding_window + batch - 1))
        else:
            caps.append(context)
    kv_bytes = sum(caps) * c.kv_heads * c.head_dim * 8
    return {"capacities": caps, "kv_bytes": kv_bytes, "state_bytes": 0, "total_bytes": kv_bytes}


def suggest_budget(file_bytes: int, mode: str) -> int:
    """context.ts:27-32 — MiB."""
    model_mib = max(0, file_bytes) / 1024 ** 2
    floor = 512 if mode == "lite" else 1024 if mode == "low-memory" else 2048
    ceiling = 1024 if mode == "lite" else 2048 if mode == "low-memory" else 6144
    return int(min(ceiling, max(floor, -(-(model_mib + 384) // 256) * 256)))


def cache_copies(start: int, count: int, capacity: int) -> list[dict]:
    """context.ts:34-37 — at most two contiguous ring writes."""
    offset = start % capacity
    first = min(count, capacity - offset)
    out = [{"source": 0, "target": offset, "count": first}]
    if first < count:
        out.append({"source": first, "target": 0, "count": count - first})
    return out
