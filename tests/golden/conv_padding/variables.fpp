#:set architecture = [('Conv', ['input'], [[1, 1], [3, 3], [2, 3, 2, 3], [1, 1]])]
#:set inputs = []
#:set trueInputs = [['input', [1, 2, 6, 6]]]
#:set outShape = [['output', [1, 3, 8, 10]]]
#:set outputs = {'output': 'input'}
