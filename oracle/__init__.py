"""CPU oracle for the qhtp B200 hot paths (TEST INFRASTRUCTURE ONLY).

This package is the parity checker, never the product.  Only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py`` may import it.  The product path
(``qcom_htp_b200``) never imports, links or executes anything here and fails
loudly when its CUDA library is missing.

Modules
-------
mm_oracle   quantized MatMul family: case generator restated from
            ``scripts/generate_qnn_matmul_python_cases.py`` and the exact
            integer/requant model (bit-exact reference for the GPU kernels).
gdn_oracle  GDN/KDA chunk triangular inverse: A generator, fp64 inverse,
            ``oc`` gate, BL=16 block model restated from
            ``example/gdn_native/solve_op/gdn_solve_ref.c``.
"""
