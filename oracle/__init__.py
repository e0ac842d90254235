"""CPU oracle and CPU baseline for the batched QR path -- test infrastructure only.

Nothing in the product package imports this directory.  ``qr_oracle`` restates
the reference algorithm in numpy (the parity checker); ``cpu_ref`` wraps the
CPU ``torch.linalg.qr`` / ``torch.geqrf`` baseline that ``bench.py`` times.
"""
