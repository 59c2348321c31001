"""Octonion (Cayley-Dickson) multiplication tables.

y_i = sum_j SIGN_TABLE[i][j] * x_j @ W[WEIGHT_IDX[i][j]], as in the reference
(src/model/constants.py:15-52).  WEIGHT_IDX[i][j] = i XOR j; the signs are
those of octonion multiplication in the reference's basis ordering.  The
tables are part of the model's definition and must match exactly.
"""

WEIGHT_IDX = [[i ^ j for j in range(8)] for i in range(8)]

SIGN_TABLE = [
    [+1, -1, -1, -1, -1, -1, -1, -1],
    [+1, +1, +1, -1, +1, -1, -1, +1],
    [+1, -1, +1, +1, +1, +1, -1, -1],
    [+1, +1, -1, +1, +1, -1, +1, -1],
    [+1, -1, -1, -1, +1, +1, +1, +1],
    [+1, +1, -1, +1, -1, +1, -1, +1],
    [+1, +1, +1, -1, -1, +1, +1, -1],
    [+1, -1, +1, +1, -1, -1, +1, +1],
]
