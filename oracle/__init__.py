"""CPU oracle for the bolt weight-streaming decode ops.

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import this
package, and only as the checker or as the timed CPU baseline.  The product
path (``nemotron_ops_b200``) never imports it and has no CPU fallback.
"""
from .bolt_oracle import *  # noqa: F401,F403
