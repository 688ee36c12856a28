"""CPU oracle for the Mote Q4_0 / per-token layer hot path.

TEST INFRASTRUCTURE ONLY: the product (``mote_b200``) never imports this
package.  ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline legs
of ``bench.py`` use it as the checker.

* ``oracle.ref`` -- ctypes bindings to ``libmote_oracle.so``, a C
  restatement of the pure-Rust ``mote-reference`` crate (bit-identical f32
  arithmetic; pinned against the reference's own known-answer tests).
* ``oracle.checker`` -- independent numpy float64 re-implementations and the
  error metrics the parity tests use.
"""
