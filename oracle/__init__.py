"""CPU oracle for scry-llm's int8 Llama decode path.

TEST INFRASTRUCTURE ONLY: the parity checker for the B200 engine and the timed
CPU baseline.  Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s
CPU-baseline / ``--impl reference`` legs may import this package.  The product
package ``esolearn_b200`` never imports it.
"""
from .oracle import *  # noqa: F401,F403
