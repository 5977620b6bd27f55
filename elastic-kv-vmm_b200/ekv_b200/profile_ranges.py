"""Optional profiler ranges around data-path calls.

With ``EKV_PROFILE_RANGES=1`` at import time the decorated callables run
inside ``torch.profiler.record_function("ekv/<name>")``, the range names the
reference uses (adaptive_sparse/profile_ranges.py:7-22); otherwise the
decorator returns the function unchanged.
"""

from __future__ import annotations

import os
from functools import wraps


def profile_range(name):
    def decorate(fn):
        if os.environ.get("EKV_PROFILE_RANGES") != "1":
            return fn

        @wraps(fn)
        def wrapped(*args, **kwargs):
            import torch

            with torch.profiler.record_function(f"ekv/{name}"):
                return fn(*args, **kwargs)

        return wrapped

    return decorate
