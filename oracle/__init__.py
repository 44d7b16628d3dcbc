"""CPU oracle of the SpikeStack Lite hot path -- test infrastructure only (see spk_oracle.py)."""
