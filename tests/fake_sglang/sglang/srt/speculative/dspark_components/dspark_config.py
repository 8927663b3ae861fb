"""DSpark's config helper (a test stand-in): gamma = draft tokens - 1."""


def dspark_gamma_from_num_draft_tokens(n: int) -> int:
    return n - 1
