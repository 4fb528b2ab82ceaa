"""CPU: the error bound behind tight binning's single-precision rows.

Tight binning sets each record's alpha ellipse up in double, reduces it to the centred
form x = cx + a Y -/+ sqrt(p Y^2 + q) (Y = y - cy) and evaluates every tile row's
x-range in float32 (diff_gabor_splatting_b200/csrc/binning.cu, record_region and
row_span), widening the range by `margin` = 2 px plus a derived bound on the float
error.  This test restates that row evaluation in numpy float32, operation for
operation (the fused multiply-add rounds once), and checks over random ellipses --
centres far from the origin, radii from 0.3 to 3000 px, anisotropy up to 300:1 -- that
the widened float range always contains the double evaluation's range widened by 2 px,
and that no tile row the double evaluation keeps is lost.  The GPU tests check the
kernels themselves (tight lists are ordered subsets of the square lists; renders are
identical with and without tight binning).
"""

import numpy as np

f32 = np.float32


def centred_form(M, cx, cy):
    """Per-record setup as the kernel does it (double): a, p, q, yl, ey, margin, yerr."""
    m00, m01, m11 = M[0, 0], M[0, 1], M[1, 1]
    k = -1.0
    a = -m01 / m00
    p = (m01 * m01 - m00 * m11) / (m00 * m00)
    q = -k / m00
    ey = np.sqrt(-q / p)
    yl = -a * np.sqrt(q / (p * (p - a * a)))
    ey_err = 2.0**-23 * (abs(cy) + ey + 64.0)
    margin = (2.0 + 2.0**-10 * np.sqrt(q) + np.sqrt(4.0 * (q / ey) * ey_err)
              + 2.0 * abs(a) * ey_err + 2.0**-20 * (abs(cx) + abs(a) * (abs(cy) + ey)))
    return a, p, q, yl, ey, margin, 2.0 * ey_err


def fma32(x, y, z):
    """float32 fused multiply-add: the exact product plus z, rounded once."""
    return f32(np.float64(x) * np.float64(y) + np.float64(z))


def test_float_rows_contain_double_rows():
    rng = np.random.default_rng(7)
    rows = 0
    min_slack = np.inf
    for _ in range(4000):
        cx, cy = rng.uniform(-3000.0, 5000.0, 2)
        r1 = 10.0 ** rng.uniform(-0.5, 3.5)
        r2 = r1 * 10.0 ** rng.uniform(-2.5, 0.0)
        th = rng.uniform(0.0, np.pi)
        R = np.array([[np.cos(th), np.sin(th)], [-np.sin(th), np.cos(th)]])
        M = R.T @ np.diag([1.0 / r1**2, 1.0 / r2**2]) @ R
        a, p, q, yl, ey, margin, yerr = centred_form(M, cx, cy)
        F = {n: f32(v) for n, v in dict(cx=cx, cy=cy, a=a, p=p, q=q, yl=yl, ey=ey,
                                         m=margin, e=yerr).items()}
        ty = np.arange(int(np.floor((cy - ey) / 16)) - 1, int(np.floor((cy + ey) / 16)) + 2)
        if len(ty) > 200:
            ty = rng.choice(ty, 200, replace=False)
        for t in ty:
            y0, y1 = 16.0 * t - 2.0, 16.0 * t + 17.0
            ya, yb = max(y0 - cy, -ey), min(y1 - cy, ey)
            if ya > yb:
                continue
            y = min(max(yl, ya), yb)
            lo = cx + a * y - np.sqrt(max(p * y * y + q, 0.0))
            y = min(max(-yl, ya), yb)
            hi = cx + a * y + np.sqrt(max(p * y * y + q, 0.0))
            # the kernel's float32 row
            fya = max(f32(f32(f32(y0) - F["cy"]) - F["e"]), -F["ey"])
            fyb = min(f32(f32(f32(y1) - F["cy"]) + F["e"]), F["ey"])
            assert fya <= fyb, "a row the double evaluation keeps was lost"
            fy = min(max(F["yl"], fya), fyb)
            d = max(fma32(f32(F["p"] * fy), fy, F["q"]), f32(0))
            flo = f32(fma32(F["a"], fy, F["cx"]) - np.sqrt(d, dtype=f32))
            fy = min(max(-F["yl"], fya), fyb)
            d = max(fma32(f32(F["p"] * fy), fy, F["q"]), f32(0))
            fhi = f32(fma32(F["a"], fy, F["cx"]) + np.sqrt(d, dtype=f32))
            slack = min((lo - 2.0) - (float(flo) - float(F["m"])),
                        (float(fhi) + float(F["m"])) - (hi + 2.0))
            min_slack = min(min_slack, slack)
            rows += 1
    assert rows > 50000
    assert min_slack >= 0.0, f"float row range short of the double range by {-min_slack} px"
