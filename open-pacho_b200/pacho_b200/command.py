"""``python -m pacho_b200``: OpenPacho's own ``pacho`` command with b200.

OpenPacho's command lists devices and runs its synchronized benchmark
(src/openpacho/cli.py:20-147); its parser offers a fixed set of backend names
(``--backend`` choices, cli.py:106 and 108).  This entry point registers b200
with OpenPacho (:func:`pacho_b200.register`), lets those two options accept
``"b200"`` as one more choice while OpenPacho builds its parser, and runs
OpenPacho's ``main`` unchanged -- the device listing, the benchmark cases,
their timing, validation and report are OpenPacho's.  Without OpenPacho
installed it exits with status 2 and says so.
"""

from __future__ import annotations

import argparse
import importlib
import sys
from contextlib import contextmanager


@contextmanager
def _backend_choice_b200():
    """While active, every ``--backend`` option built with a ``choices``
    list also accepts ``"b200"``."""
    original = argparse._ActionsContainer.add_argument

    def add_argument(self, *names, **kwargs):
        choices = kwargs.get("choices")
        if "--backend" in names and choices is not None and "b200" not in choices:
            kwargs["choices"] = (*choices, "b200")
        return original(self, *names, **kwargs)

    argparse._ActionsContainer.add_argument = add_argument
    try:
        yield
    finally:
        argparse._ActionsContainer.add_argument = original


def main(argv=None, openpacho=None) -> int:
    if openpacho is None:
        try:
            import openpacho  # type: ignore[import-not-found]
        except ImportError:
            print("pacho_b200: OpenPacho is not installed; the pacho command is OpenPacho's "
                  "(pip install open-pacho), b200 plugs into it", file=sys.stderr)
            return 2
    from .register import register

    register(openpacho)
    cli = importlib.import_module(openpacho.__name__ + ".cli")
    with _backend_choice_b200():
        return cli.main(argv)
