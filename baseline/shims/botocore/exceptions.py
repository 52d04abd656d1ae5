"""Exception names that ``olmo.util`` refers to at import time."""


class BotoCoreError(Exception):
    pass


class ClientError(BotoCoreError):
    pass


class HTTPClientError(BotoCoreError):
    pass


class ConnectionError(BotoCoreError):
    pass


def __getattr__(name):
    # any other exception class the reference names resolves to a distinct subclass
    if name[:1].isupper():
        cls = type(name, (BotoCoreError,), {})
        globals()[name] = cls
        return cls
    raise AttributeError(name)
