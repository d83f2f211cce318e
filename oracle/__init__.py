"""CPU oracle for the quantized DiT-block hot path.

TEST INFRASTRUCTURE ONLY. Nothing in the product package (``h3b200``) imports,
links or executes anything under this directory. Only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference`` legs
of ``bench.py`` may use it, and only as the checker or as the timed CPU
baseline -- never as the thing measured or shipped.

Parity pin: every function here is checked against golden vectors produced by
running the reference's own eager implementation (comfy_kitchen 0.2.28, vendored
in X-MinimaxH3 under ``backends/turbo/vendor/comfy_kitchen``) in a container
where the reference is importable. The vectors and the script that made them
live in ``tests/golden/``.
"""

from .h3_oracle import *  # noqa: F401,F403
