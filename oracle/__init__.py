"""Test infrastructure: the CPU oracle of the attention path (see ``oracle/attention.py``).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline legs may import this package. The product
package ``ebr_b200`` never does.
"""

from oracle import attention

__all__ = ["attention"]
