"""Drop-in tree with the reference's import paths (``src.kernels.*``,
``src.agents.mappo``) over the tarmac_b200 sm_100a kernels."""
