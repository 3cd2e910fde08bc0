def PRNGKey(seed):
    return seed
