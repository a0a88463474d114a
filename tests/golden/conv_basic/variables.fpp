#:set architecture = [('Conv', ['input'], [[1, 1], [3, 3], [0, 0, 0, 0], [1, 1]])]
#:set inputs = []
#:set trueInputs = [['input', [2, 2, 7, 7]]]
#:set outShape = [['output', [2, 3, 5, 5]]]
#:set outputs = {'output': 'input'}
