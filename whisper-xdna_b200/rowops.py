"""Drop-in for the reference's src/rowops.py: the same design functions, on the
B200 (see wxb200.rowops)."""
from wxb200.rowops import *  # noqa: F401,F403
from wxb200.rowops import (gelu_row, gelu_row2, gelu_row3, gelu_row4,  # noqa: F401
                           gelu_row4_rne, gelu_row4f, layer_norm, layer_norm_gb,
                           softmax_row, softmax_row2, softmax_row3, softmax_row3_win,
                           softmax_row4, softmax_row4_win, softmax_row4r_win, softmax_rows)
