class SchemeClient:
    recoverable_errors = ()
    scheme = ""

    def __init__(self, resource=None):
        self.resource = resource


def add_scheme_client(client):
    return None
