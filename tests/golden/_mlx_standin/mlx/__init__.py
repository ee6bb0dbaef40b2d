"""Stand-in for the ``mlx`` package, used only by ``tests/golden/make_golden.py``.

MLX (``pyproject.toml:32`` of the reference: ``mlx>=0.22.0``) cannot be
installed in this container. This stand-in implements the handful of
``mlx.core`` array primitives that the reference's pure per-step functions,
its v2 test bodies and its parity helper call, on top of torch float64, so
that the reference's own Python code can run here and emit golden vectors.
"""
