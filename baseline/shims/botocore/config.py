class Config:
    def __init__(self, *a, **k):
        pass
