"""`python -m sejong_b200 <command>`: the train / train-value / benchmark / init / inspect / generate
commands (sejong_b200/cli.py)."""
import sys

from .cli import main

sys.exit(main())
