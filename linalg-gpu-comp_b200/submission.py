"""Drop-in replacement for the reference's submission.py (GPU MODE ``qr`` task).

Place this directory on ``sys.path`` (or run the harness from it) and the
reference harness (reference_repo/eval.py:126, 184 ``from submission import
custom_kernel``) calls the B200 library: ``custom_kernel(data) -> (H, tau)`` in
torch.geqrf compact form.
"""
from qr_b200 import custom_kernel  # noqa: F401
