#:set architecture = [('Conv', ['input'], [[1, 1], [3, 3], [0, 0, 0, 0], [2, 2]])]
#:set inputs = []
#:set trueInputs = [['input', [1, 2, 7, 7]]]
#:set outShape = [['output', [1, 3, 3, 3]]]
#:set outputs = {'output': 'input'}
