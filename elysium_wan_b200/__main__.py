"""python -m elysium_wan_b200 <subcommand> ... (the `wantrain` CLI)."""

import sys

from elysium_wan_b200.cli import main

sys.exit(main())
