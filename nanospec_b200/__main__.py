"""``python -m nanospec_b200 ...``: the training CLI (see ``nanospec_b200.cli``)."""

from .cli import main

main()
