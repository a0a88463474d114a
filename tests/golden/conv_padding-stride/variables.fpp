#:set architecture = [('Conv', ['input'], [[1, 1], [3, 3], [2, 3, 2, 3], [2, 2]])]
#:set inputs = []
#:set trueInputs = [['input', [1, 2, 6, 6]]]
#:set outShape = [['output', [1, 3, 4, 5]]]
#:set outputs = {'output': 'input'}
