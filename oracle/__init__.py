"""CPU oracle for the continuous-batching forward step (TEST INFRASTRUCTURE).

A numpy restatement of the reference's algorithms (Complexity-ML/
complexity-inference, package ``mu_inference``), used only as the checker:
by ``tests/``, by ``__graft_entry__.smoke()`` and by the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py``.  The product path
(``complexity-inference_b200/mu_b200``) never imports anything from here.

Parity pin: the oracle is checked against golden vectors produced by running
the reference itself on this container's CPU (``tests/golden/make_golden.py``
and the fixtures next to it); see ``tests/test_oracle_golden.py``.
"""

from .mu_oracle import *  # noqa: F401,F403
