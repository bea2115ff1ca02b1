"""The CPU oracle: numpy restatements of the reference's attention and
acceptance step. TEST INFRASTRUCTURE ONLY: imported by tests/, by
__graft_entry__.smoke() as the checker, and by bench.py's CPU legs. The
product package wpt_b200 never imports it."""

from . import accept, attention  # noqa: F401
