"""CPU oracle for the block-sparse attention path.

Test infrastructure: only ``tests/``, ``__graft_entry__.smoke()`` and the
CPU-baseline leg of ``bench.py`` may use it, and only as the checker. The
``sabrecoder_b200`` package never imports it.

Parity of this oracle is pinned against golden fixtures recorded from the
reference implementation itself (see ``tests/golden/gen_golden.py``).
"""

from . import attention_oracle, mask_oracle  # noqa: F401
