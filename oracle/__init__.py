"""CPU oracle for the Hyena FFT-conv hot path — TEST INFRASTRUCTURE ONLY.

Nothing in the product package (``nvsubquadratic_b200``) imports this package.
Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` may import it, and there only as the checker (or, for the CPU
baseline, as the timed stand-in for the reference's own CPU path).

Contents
--------
``fftconv``  restatement of nvSubquadratic's ``nvsubquadratic/ops/fftconv.py``
             (zero-padded linear FFT convolution, 1D causal / 1D / 2D / 3D,
             BHL and BLH layouts, optional ``shortcut`` D-skip) written as one
             generic N-D routine over ``torch.fft`` on the CPU (the same
             library the reference calls), so it is differentiable and can be
             timed as the reference's CPU path.
``direct``   independent float64 numpy direct (spatial) convolution used to
             check the FFT restatement itself on tiny shapes.
``hyena``    restatement of the Hyena mixer composition
             (``nvsubquadratic/modules/hyena_nd.py:497-583``) for identity
             norms, with the depthwise short conv semantics of
             ``modules/distributed_depthwise_conv_nd.py`` / ``causal_conv1d.py``.
``cp``       restatement of the context-parallel all-to-all redistribution and
             zigzag chunk layout (``nvsubquadratic/parallel/a2a_comms.py``,
             ``nvsubquadratic/parallel/utils.py:122-206``) as single-process
             index arithmetic over per-rank tensors.

Pinning: every function here is checked against golden vectors produced by
running the reference itself (``tests/golden/make_golden.py``, fixtures in
``tests/golden/*.pt``) in ``tests/test_oracle_golden.py``.
"""
