"""CPU checkers for the B200 spectral backend (test infrastructure only).

spectral_oracle: numpy restatement of the reference algorithm.
ref_runner:      the reference itself, compiled from its sources (oracle/_ref).
"""
