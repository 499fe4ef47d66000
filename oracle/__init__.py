"""CPU oracle for the FP8-checkpoint + replay GDN decode path.

TEST INFRASTRUCTURE ONLY.  Nothing in the product package imports this
directory.  Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline
leg of ``bench.py`` may use it, and there only as the checker / the timed CPU
baseline, never as the thing measured for the GPU path.

The oracle is a numpy restatement of the reference prototype's algorithm:

* ``prototype/gdn_replay_fp8_reference.py`` (zz774ever/fp8-replayssm-gdn-kernel)
  for the FP8/INT8 codec, the per-token recurrence and the replay chain;
* ``prototype/gdn_replayssm_fp8_kernel.py`` for the prep stage (q/k L2 norm,
  gating, ring append) and the backward ("adjoint") replay form.

Parity is pinned by ``tests/golden/*.npz`` which were produced by importing
the reference module itself on CPU (``tests/golden/make_golden.py``).
"""

from .gdn_oracle import *  # noqa: F401,F403
