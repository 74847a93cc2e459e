"""The split decode's work ranges on CPU: CTA c of G owns page-groups [floor(c P / G),
floor((c + 1) P / G)). The kernels (localstack_b200/csrc/decode.cuh, range_lo / cta_of) compute
the floor in double precision - one correctly rounded multiply (exact, the product is below 2^53)
and one correctly rounded divide - on the argument that a non-integer quotient lies at least 1/G
below the next integer, more than half an ulp of any value below 2^42 while G < 4096. Python
floats are the same IEEE doubles with the same two operations, so this checks the argument over
the whole range the kernels allow (G <= 512 CTAs, P below 2^31 page-groups)."""
import numpy as np

K_MAX_CTAS = 512


def range_lo_double(c, P, G):
    return int(float(c) * float(P) / float(G))


def range_lo_exact(c, P, G):
    return (c * P) // G


def cta_of_double(x, P, G):
    # the kernel's search: a double-precision first guess, then integer steps on range_lo
    c = int(float(x) * float(G) / float(P))
    while c + 1 < G and range_lo_double(c + 1, P, G) <= x:
        c += 1
    while c > 0 and range_lo_double(c, P, G) > x:
        c -= 1
    return c


def test_range_lo_double_is_exact_on_edges_and_random_cases():
    rng = np.random.default_rng(0)
    cases = []
    for G in (1, 2, 3, 7, 34, 147, 148, 160, 255, 256, 296, 511, 512):
        for P in (1, 2, G - 1 if G > 1 else 1, G, G + 1, 4096, 65535, 2 ** 20 + 1, 2 ** 31 - 1, 2 ** 31 - 2,
                  int(rng.integers(1, 2 ** 31))):
            if P <= 0:
                continue
            for c in (0, 1, G // 2, G - 1, G):
                cases.append((c, P, G))
    for _ in range(200000):
        G = int(rng.integers(1, K_MAX_CTAS + 1))
        P = int(rng.integers(1, 2 ** 31))
        c = int(rng.integers(0, G + 1))
        cases.append((c, P, G))
    for c, P, G in cases:
        assert range_lo_double(c, P, G) == range_lo_exact(c, P, G), (c, P, G)


def test_cta_of_finds_the_owning_range():
    rng = np.random.default_rng(1)
    for _ in range(3000):
        G = int(rng.integers(1, K_MAX_CTAS + 1))
        P = int(rng.integers(1, 2 ** 31)) if rng.random() < 0.5 else int(rng.integers(1, 4 * G))
        x = int(rng.integers(0, P))
        c = cta_of_double(x, P, G)
        lo, hi = range_lo_exact(c, P, G), range_lo_exact(c + 1, P, G)
        assert lo <= x < hi, (x, P, G, c)
