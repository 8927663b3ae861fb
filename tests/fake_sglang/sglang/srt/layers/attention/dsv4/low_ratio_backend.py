"""SGLang's decode-indexer decisions (a test stand-in: set ``IDENTITY`` / ``FITS``)."""

IDENTITY = False
FITS = False


def low_ratio_decode_rows_are_identity(*, backend, forward_batch, ratio):
    return IDENTITY


def low_ratio_decode_rows_fit_candidate_span(*, backend, forward_batch):
    return FITS
