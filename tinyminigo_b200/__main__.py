"""`python -m tinyminigo_b200 ...`: the reference's command line (src/main.rs)."""
import sys

from .cli import main

sys.exit(main())
