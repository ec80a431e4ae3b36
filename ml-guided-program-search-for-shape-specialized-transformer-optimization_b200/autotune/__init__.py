"""Program search over the sm100 kernel variants.

``search_space`` mirrors the reference's ``autotune.search_space`` surface
(ProgramSearchSpace and friends) over the kernels built into libb200tx;
``sweep`` times every candidate of a space on the GPU and publishes the
fastest into the deployment registry.  The reference's Optuna loop, study
storage and evidence bookkeeping are not part of this package.
"""
