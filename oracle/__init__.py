"""CPU oracle for the YABT per-tree growth path -- TEST INFRASTRUCTURE ONLY.

This package restates, in numpy (plus one C file compiled from the reference's
own source for the timed CPU baseline), the algorithm of grafael/yabt's GPU
tree-growth path so that the CUDA implementation in ``yabt_b200`` can be
checked against it. Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU
legs of ``bench.py`` may import it, and only as the checker or as the timed
CPU baseline -- never as a code path of the product. ``yabt_b200`` itself
never imports this package and has no CPU fallback.

Every function cites the reference file:line it restates (paths relative to
the reference project's root). Parity is pinned against golden vectors
produced by running the reference itself (``tests/golden/make_golden.py``).

Modules
-------
binning   Binner.fit / transform / impute / edge_value   (yabt/binning.py)
grow      level-wise grower, histograms, split scan      (yabt/tree.py, yabt/histogram.py)
leafnet   ridge-linear neural leaves                     (yabt/neural_leaves.py)
boost     losses, interaction detector, boosting loop    (yabt/boosting.py, yabt/adaptive_features.py)
cgrow     ctypes binding of the reference's own OpenMP C grower (yabt/_cgrow/grow.c),
          compiled from the reference sources into oracle/_ref/ (CPU baseline)
"""
