"""TEST INFRASTRUCTURE ONLY.

CPU restatement of the nsa-hopper reference's selected-branch forward, used as the checker by
tests/, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm.  The
product (the sm_100a kernel behind include/nsa_sel.h) never imports or calls it.
"""
from .oracle import build, count_keys, default_threads, forward, forward_window  # noqa: F401
