# SPDX-License-Identifier: Apache-2.0
"""Entry for Python child processes started with ``spawn``.

A spawned interpreter does not run vLLM's plugin discovery, so a host that
starts workers itself passes ``child_entry`` as the process target with its own
target as the first argument: the codec registers (subject to the same
environment switches as ``plugin.register``) before the host target runs.
Same contract as the reference's src/gdn_state_codec/bootstrap.py:9-15.
"""

from __future__ import annotations

from typing import Any, Callable


def child_entry(target: Callable[..., Any], *args: Any, **kwargs: Any) -> Any:
    from .plugin import register

    register()
    return target(*args, **kwargs)


__all__ = ["child_entry"]
