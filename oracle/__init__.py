"""CPU oracle for the kvcompress JoLT / FlashJoLT compress/decompress path.

TEST INFRASTRUCTURE ONLY.  Nothing in ``kvcompress_b200`` imports this
package.  It is imported by ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` -- always as
the checker or as the timed CPU baseline, never as the thing measured or
shipped.

The oracle is a numpy restatement of the reference algorithm
(sachncs/kvcompress, ``kvcompress/compressor/*.py``); every function cites
the reference file:line it follows.  Random inputs (the JL matrix and the
randomised-SVD sketch) are *arguments*: the reference draws them from
torch's own generators, and the tests draw them the same way and hand the
arrays in.

Parity pin: ``tests/test_oracle_golden.py`` checks this module against the
golden vectors in ``tests/golden/`` that ``tests/golden/make_golden.py``
produced by running the reference itself.
"""

from oracle.jolt import *  # noqa: F401,F403
