"""CPU oracle for the BS-RoFormer / Mel-band RoFormer training hot path.

TEST INFRASTRUCTURE ONLY.  Nothing in the product package (``pymsst_b200``)
imports this package; only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` use it, and only
as the checker or the timed CPU baseline.

Contents
--------
``ops_ref``      restatements of the reference's fused-kernel formulas
                 (src/pymsst/training/cuda/fused_band_split.cu), computed in
                 the input dtype (float64 inputs give a float64 reference).
``mel_ref``      the Slaney mel filterbank and the Mel-band index tables
                 (librosa.filters.mel algorithm, float64), plus the gather /
                 scatter-add-average recombination of pymss-core's
                 MelBandRoformer.
``roformer_ref`` a pure-PyTorch restatement of pymss-core 0.1.4's BSRoformer
                 and MelBandRoformer (same constructor arguments, forward and
                 state-dict keys), used as the model-level oracle and as the
                 CPU baseline.
``audio_ref``    the seeded synthetic stereo audio generator of the
                 benchmark configurations, and the training loss.

Pinning
-------
* Kernel formulas: pinned against outputs of the reference's own CUDA
  extension, compiled from its sources by ``oracle/build_ref.py`` into
  ``oracle/_ref/`` and run once on a B200; the vectors are committed under
  ``tests/golden/`` with the script that produced them.
* Mel tables: pinned against torchaudio's independent Slaney filterbank.
* Model level: pymss-core 0.1.4 (the package that holds the reference model
  code) is not installed and not vendored in the reference, so the model
  restatement is parity-UNPINNED against pymss-core itself; it follows the
  reference's call sites and tests (src/pymsst/training/fused_roformer.py,
  tests/test_training_smoke.py) and the published BS-RoFormer /
  Mel-band RoFormer architecture.
"""
