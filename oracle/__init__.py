"""CPU oracle (numpy restatement of the reference's checking arithmetic) - test infrastructure only."""
from .oracle import *  # noqa: F401,F403
