"""Makes the reference package ``qwenquest`` importable for the tests, the benchmark and the smoke run.

The B200 backends plug into the reference: they subclass its
``AttentionBackend`` and use its pools, ``ForwardBatch`` and config parser, so
whatever runs them needs ``qwenquest`` on the path.  Looked up in order: an
already importable ``qwenquest``; the directory named by ``QWENQUEST_REF``
(one that holds the ``qwenquest`` package); ``baseline/_ref`` in this
repository (``pip install --no-deps --target baseline/_ref <reference>``,
which ``__graft_entry__.build()`` performs when the reference source is
present).
"""

from __future__ import annotations

import importlib.util
import os
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parents[1]
INSTALL_DIR = REPO / "baseline" / "_ref"


def candidates() -> list[Path]:
    out = []
    env = os.environ.get("QWENQUEST_REF")
    if env:
        out.append(Path(env))
    out.append(INSTALL_DIR)
    return out


def ensure_importable() -> None:
    if importlib.util.find_spec("qwenquest") is not None:
        return
    for cand in candidates():
        if (cand / "qwenquest" / "__init__.py").exists():
            sys.path.insert(0, str(cand))
            return
    raise ImportError(
        "the reference package `qwenquest` is not importable: install it with "
        "`pip install --no-deps --target baseline/_ref <QwenQuest checkout>` or set QWENQUEST_REF to a "
        "directory that holds it")


def available() -> bool:
    try:
        ensure_importable()
    except ImportError:
        return False
    return True
