"""CPU oracle for the EWS hot path: TEST INFRASTRUCTURE ONLY.

This package is a float64 (or float32) restatement, on the CPU with torch, of the reference's
algorithm for the EWS layer (alexandre-bloch/exponentially-weighted-signature): the series /
plane / block-series local terms, the modified-Chen packed operator, its associative prefix scan
and power-of-two terminal tree, the layer's readouts, and the log-signature epilogue. Gradients
come from torch autograd, as the reference's come from JAX autodiff.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may import it,
and only as the checker (or, for ``bench.py --impl reference``, as the timed stand-in for the
reference's jax[cpu] path, which cannot be installed on these machines). The product path in
``exponentially_weighted_signature_b200`` never imports it and has no CPU fallback.

Parity pins (``tests/test_oracle_pins.py``): the reference's analytic known answers (depth one
equals the augmented-exponential affine recursion, A = 0 gives the classical signature,
exp(log(EWS)) = EWS, engine cross-agreement of the closed-form leaves with the series leaf,
associative scan = sequential recursion, the series error bound, Witt dimensions, finite
differences). The reference's own golden files (``tests/reference_kernel_outputs.npz``) rebuild
their model from JAX's threefry PRNG and exercise the default Van Loan leaf, so they cannot be
reproduced without JAX. The Lyndon compression order of the log-signature follows signax 0.2.1's
published definition (coefficients of the Lyndon words, Duval order) and is parity-unpinned.
"""
