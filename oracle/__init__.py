"""CPU oracle for the AIOS-IME CandidateGroup hot path — TEST INFRASTRUCTURE ONLY.

A restatement, in numpy / CPU torch, of the reference algorithms this repository
replaces with sm_100a kernels (7155/aios, paths cited per function). It is the
checker used by ``tests/``, by ``__graft_entry__.smoke()`` and by the CPU baseline
legs of ``bench.py``; the product package ``aios_b200`` never imports it.

Pinning: ``tests/test_oracle_golden.py`` checks every function here against
golden fixtures produced by running the unmodified reference code on CPU
(``tests/golden/make_golden.py``).
"""
