class OmegaConfBaseException(Exception):
    pass
